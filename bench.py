"""Benchmark: MacBoost batch inference on B200 (rows*trees per second).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg2]
                    [--impl ours|reference] [--scaling weak|strong]

One process per GPU (torchrun for N > 1; RANK / LOCAL_RANK / WORLD_SIZE from
the environment).  A step is one predict over the rank's whole row shard of
the configuration (BASELINE.json configs[1] by default: 10M rows x 28
features, 100 depth-6 trees, fused sigmoid output).  Rows shard with no
collective on the data path; torch.distributed (gloo, CPU tensors) is used
only for the barriers and the max-over-ranks of the timings.

Scaling (the configs' own splits): cfg1-cfg4 are strong-scaled -- the
config's rows are split into N contiguous shards; cfg5 runs proportional
slices -- 50M / 8 rows per GPU, so N GPUs predict N/8 of the 50M rows (weak).

value  -- device-resident input: K launches timed with CUDA events on the
          launching stream, max over ranks.
e2e    -- the reference-facing C-ABI call (macboost_predict_ex) on page-locked
          host buffers: host->device copy, kernel and device->host copy of the
          outputs inside the timed region, max over ranks.
cpu_baseline -- the oracle (C restatement of the reference CPU predictor,
          all host threads) on a bounded prefix of the timed rows, rank 0,
          N == 1 only; the same leg compares those rows' GPU outputs with the
          oracle's ("parity": raw margins bit for bit, the step's transformed
          output within 2 ulp).  When the reference's own Python package is
          installed in baseline/_ref, its numpy predictor (PyModel.predict_raw)
          is timed beside it ("cpu_baseline_reference").
e2e_copy_ceiling -- plain page-locked H2D and D2H copies of the same bytes as
          an e2e step, timed with CUDA events while every rank copies at once
          (max over ranks): the host-link bound of the e2e number.
--impl reference -- times that CPU predictor as the reference arm.
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
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from macboost_b200 import synth  # noqa: E402

METRIC = json.loads((ROOT / "BASELINE.json").read_text())["metric"] \
    if (ROOT / "BASELINE.json").exists() else "predict rows·trees/s"
UNIT = "rows·trees/s"
OUTPUT_KIND = {"raw": 1, "sigmoid": 2, "softmax": 2}


def _env_int(name, default):
    try:
        return int(os.environ.get(name, default))
    except ValueError:
        return default


class Dist:
    """Barrier and max-over-ranks over gloo (control plane only)."""

    def __init__(self):
        self.rank = _env_int("RANK", 0)
        self.world = _env_int("WORLD_SIZE", 1)
        self.local_rank = _env_int("LOCAL_RANK", 0)
        self.pg = None
        if self.world > 1:
            import datetime

            import torch.distributed as dist
            dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
            self.dist = dist

    def barrier(self):
        if self.world > 1:
            self.dist.barrier()

    def max(self, v: float) -> float:
        if self.world == 1:
            return v
        import torch
        t = torch.tensor([float(v)], dtype=torch.float64)
        self.dist.all_reduce(t, op=self.dist.ReduceOp.MAX)
        return float(t.item())

    def close(self):
        if self.world > 1:
            self.dist.destroy_process_group()


class ClockSampler:
    """SM clocks and clock-event (throttle) reasons during the timed region.

    NVML, read by a thread every 5 ms, plus `sample()` calls that the timed
    loop makes while its queued launches are still running, so that even a
    region of a few milliseconds holds samples.  Falls back to nvidia-smi
    (50 ms) when NVML cannot be opened."""

    REASONS = (("hw_slowdown", "nvmlClocksEventReasonHwSlowdown", 0x8),
               ("hw_thermal_slowdown", "nvmlClocksEventReasonHwThermalSlowdown", 0x40),
               ("sw_thermal_slowdown", "nvmlClocksEventReasonSwThermalSlowdown", 0x20),
               ("sw_power_cap", "nvmlClocksEventReasonSwPowerCap", 0x4))
    SMI_FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
                  "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
                  "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device: int):
        self.device = device
        self.samples = []          # (sm MHz, set of reasons)
        self.max_mhz = None
        self.nvml = None
        self.handle = None
        self.proc = None
        self.lines = []
        self.running = False
        self.lock = threading.Lock()
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nvml = pynvml
            self.handle = self._nvml_handle(device)
            self.max_mhz = float(pynvml.nvmlDeviceGetMaxClockInfo(self.handle,
                                                                 pynvml.NVML_CLOCK_SM))
            self._reason_fn = getattr(pynvml, "nvmlDeviceGetCurrentClocksEventReasons", None) \
                or pynvml.nvmlDeviceGetCurrentClocksThrottleReasons
        except Exception:
            self.nvml = None

    def _nvml_handle(self, device):
        pynvml = self.nvml
        try:
            import torch
            uuid = str(torch.cuda.get_device_properties(device).uuid)
            return pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
        except Exception:
            return pynvml.nvmlDeviceGetHandleByIndex(device)

    def sample(self):
        if self.nvml is None:
            return
        try:
            mhz = float(self.nvml.nvmlDeviceGetClockInfo(self.handle, self.nvml.NVML_CLOCK_SM))
            mask = int(self._reason_fn(self.handle))
        except Exception:
            return
        active = {name for name, attr, bit in self.REASONS
                  if mask & int(getattr(self.nvml, attr, bit))}
        with self.lock:
            self.samples.append((mhz, active))

    def _loop(self):
        while self.running:
            self.sample()
            time.sleep(0.005)

    def start(self):
        if self.nvml is not None:
            self.running = True
            self.thread = threading.Thread(target=self._loop, daemon=True)
            self.thread.start()
            return
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.SMI_FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50", "-i", str(self.device)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except (OSError, ValueError):
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read_smi, daemon=True)
        self.thread.start()

    def _read_smi(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def stop(self) -> dict | None:
        if self.nvml is not None:
            self.running = False
            self.thread.join(timeout=2)
        elif self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
            self.thread.join(timeout=2)
            for ln in self.lines:
                parts = [p.strip() for p in ln.split(",")]
                if len(parts) < 9:
                    continue
                try:
                    mhz = float(parts[1])
                    self.max_mhz = float(parts[2])
                except ValueError:
                    continue
                active = {name for (name, _, _), v in zip(self.REASONS, parts[5:9])
                          if v.lower().startswith("active")}
                self.samples.append((mhz, active))
        else:
            return None
        if not self.samples:
            return None
        reasons = set().union(*(r for _, r in self.samples))
        return {"sm_mhz": statistics.median(m for m, _ in self.samples),
                "sm_max_mhz": self.max_mhz, "reasons": sorted(reasons),
                "samples": len(self.samples), "source": "nvml" if self.nvml else "nvidia-smi"}


def bind_near_gpu(device: int) -> str | None:
    """Restrict this rank's threads to the CPU cores NVML reports as closest to
    `device`, so that page-locked host buffers allocated afterwards land in that
    socket's memory (first touch) and the host-device copies stay off the
    inter-socket link.  Used for N > 1; returns the core list, or None."""
    try:
        import pynvml
        import torch
        pynvml.nvmlInit()
        uuid = str(torch.cuda.get_device_properties(device).uuid)
        h = pynvml.nvmlDeviceGetHandleByUUID(("GPU-" + uuid).encode())
        ncpu = os.cpu_count() or 1
        words = pynvml.nvmlDeviceGetCpuAffinity(h, (ncpu + 63) // 64)
        cpus = {64 * w + b for w, m in enumerate(words) for b in range(64) if (m >> b) & 1}
        cpus &= os.sched_getaffinity(0)
        if not cpus:
            return None
        os.sched_setaffinity(0, cpus)
        return f"{min(cpus)}-{max(cpus)} ({len(cpus)} cores)"
    except Exception:
        return None


def traffic_lookup(cfg: str):
    """DRAM bytes per row measured by ncu for `cfg` (profiles/traffic_per_row.txt)."""
    p = ROOT / "profiles" / "traffic_per_row.txt"
    if not p.exists():
        return None
    for line in p.read_text().splitlines():
        parts = line.split()
        if len(parts) >= 2 and not line.startswith("#") and parts[0] == cfg:
            try:
                return {"bytes_per_row": float(parts[1])}
            except ValueError:
                return None
    return None


def measured_peak_hbm():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (ValueError, KeyError, OSError):
            pass
    return 6650.0, "fallback"


def cpu_baseline(cfg, text, X, budget_s=10.0, threads=None):
    """Oracle (C restatement of predictCPU) on a bounded prefix of the timed
    rows X (feature-major, F x rows).  Returns the baseline and the oracle's
    raw margins of those rows (the parity check's reference)."""
    from oracle import oracle as O
    O.build()
    om = O.model_from_dict(json.loads(text))
    nt = threads or os.cpu_count() or 1
    rows_total = X.shape[1]
    probe = min(rows_total, 20_000)
    t0 = time.perf_counter()
    O.predict_raw(om, X[:, :probe], layout="feature", nthreads=nt)
    dt = max(time.perf_counter() - t0, 1e-6)
    n = int(min(rows_total, max(probe, probe * budget_s / dt)))
    Xs = np.ascontiguousarray(X[:, :n])
    t0 = time.perf_counter()
    raw = O.predict_raw(om, Xs, layout="feature", nthreads=nt)
    dt = time.perf_counter() - t0
    return {"value": n * cfg.trees / dt, "unit": UNIT, "cores": nt, "kind": "port",
            "sample": f"the first {n} of the timed rows of {cfg.name} x {cfg.trees} trees, "
                      f"{dt:.2f} s, {nt} threads (oracle/mbref.c, restatement of "
                      f"Booster.swift predictCPU)"}, raw, om


def parity_check(O, om, raw_o, raw_gpu, out_gpu, kind, leaf_o=None):
    """The timed step's outputs of the rows the oracle scored, against it."""
    n = raw_o.shape[0]
    raw_bitwise = bool(np.array_equal(np.ascontiguousarray(raw_gpu[:n]).view(np.uint32),
                                      np.ascontiguousarray(raw_o).view(np.uint32)))
    if kind == 3:
        same = bool(np.array_equal(out_gpu[:n], leaf_o))
        return {"rows": int(n), "raw_bitwise": raw_bitwise, "leaf_indices_equal": same,
                "against": "oracle/mbref.c (restatement of Booster.swift predictCPU, pinned to "
                           "the reference's PyModel outputs in tests/golden)"}
    if kind == 2:
        want = O.predict_proba(raw_o if om.num_classes > 1 else raw_o[:, 0]).astype(np.float32)
    else:
        want = raw_o
    got = np.ascontiguousarray(out_gpu[:n], dtype=np.float32)
    ulp = int(O.ulp_distance(got, want).max()) if n else 0
    return {"rows": int(n), "raw_bitwise": raw_bitwise, "output_max_ulp": ulp,
            "output_within_2_ulp": ulp <= 2,
            "against": "oracle/mbref.c (restatement of Booster.swift predictCPU, pinned to "
                       "the reference's PyModel outputs in tests/golden)"}


def reference_pymodel(cfg, text, X, budget_s=10.0):
    """The reference's own CPU predictor, PyModel.predict_raw
    (python/macboost/_pyinfer.py:52-72), imported unmodified from the package
    installed in baseline/_ref, timed on a bounded prefix of the timed rows;
    None when that package is not installed on this machine."""
    ref = ROOT / "baseline" / "_ref"
    if not (ref / "macboost" / "_pyinfer.py").exists():
        return None
    import importlib.util
    import tempfile
    spec = importlib.util.spec_from_file_location("_mb_ref_pyinfer",
                                                  ref / "macboost" / "_pyinfer.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    with tempfile.NamedTemporaryFile("w", suffix=".json", delete=False) as fh:
        fh.write(text)
        path = fh.name
    try:
        pm = mod.PyModel(path)
    finally:
        os.unlink(path)
    probe = min(X.shape[1], 2_000)
    t0 = time.perf_counter()
    pm.predict_raw(np.ascontiguousarray(X[:, :probe].T))
    dt = max(time.perf_counter() - t0, 1e-6)
    n = int(min(X.shape[1], max(probe, probe * budget_s / dt)))
    Xr = np.ascontiguousarray(X[:, :n].T)
    t0 = time.perf_counter()
    pm.predict_raw(Xr)
    dt = time.perf_counter() - t0
    return {"value": n * cfg.trees / dt, "unit": UNIT, "cores": 1, "kind": "reference",
            "sample": f"the first {n} of the timed rows x {cfg.trees} trees, {dt:.2f} s; "
                      f"PyModel.predict_raw (numpy, one process) from the reference package "
                      f"installed unmodified in baseline/_ref; host has {os.cpu_count()} cores"}


def run_reference(args, dist, cfg, text):
    """--impl reference: the reference CPU predictor (restated) on host cores."""
    if dist.rank != 0:
        return None
    from oracle import oracle as O
    O.build()
    om = O.model_from_dict(json.loads(text))
    nt = os.cpu_count() or 1
    n = min(cfg.rows, args.ref_rows)
    X = synth.make_data(cfg, rows=n, layout="feature", seed=cfg.data_seed + 99)
    for _ in range(args.warmup):
        O.predict_raw(om, X[:, : min(n, 4096)], layout="feature", nthreads=nt)
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        O.predict_raw(om, X, layout="feature", nthreads=nt)
        times.append(time.perf_counter() - t0)
    dt = sum(times)
    value = n * cfg.trees * args.steps / dt
    return {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": 1e3 * dt / args.steps, "higher_is_better": True,
            "scaling": args.scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded)", "config": config_block(cfg, n, args),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": nt, "kind": "port",
                             "sample": f"{n} rows of {cfg.name} per step x {cfg.trees} trees"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0,
                    "d2h_bytes_per_step": 0}}


def default_scaling(cfg) -> str:
    """cfg5 runs proportional slices (50M / 8 rows per GPU); the others split
    the config's rows over the GPUs."""
    return "weak" if cfg.name == "cfg5" else "strong"


def rows_per_rank(cfg, args, world) -> int:
    if args.rows:
        rows = args.rows
    elif args.scaling == "weak":
        rows = cfg.rows // 8 if cfg.name == "cfg5" else cfg.rows
    else:
        rows = cfg.rows // world
    return (rows + 3) // 4 * 4


def config_block(cfg, rows_per_rank, args):
    split = ("proportional slices: 50M / 8 rows per GPU" if cfg.name == "cfg5"
             and args.scaling == "weak" else
             f"{args.scaling} scaling: the config's rows split over the GPUs"
             if args.scaling == "strong" else f"{args.scaling} scaling")
    return {"workload": f"{cfg.name}: {cfg.data}; model: {cfg.model}",
            "rows_per_gpu": rows_per_rank, "features": cfg.features, "trees": cfg.trees,
            "classes": cfg.classes, "output": cfg.output, "parallelism": "row shards",
            "split": split,
            "l2": "inputs larger than L2 (each step reads every row once)"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--config", default="cfg2")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--scaling", default=None, choices=["weak", "strong"],
                    help="default: strong for cfg1-cfg4, proportional slices (weak) for cfg5")
    ap.add_argument("--rows", type=int, default=0, help="override rows per GPU")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--ref-rows", type=int, default=200_000)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--workload", default="predict", choices=["predict", "contrib", "binned"],
                    help="predict: the headline (forest predict); contrib: TreeSHAP "
                         "contributions; binned: one tree walked over binned rows per step, "
                         "as a trainer evaluates each new tree, plus bin_data")
    ap.add_argument("--trees", type=int, default=0, help="override the model's tree count")
    ap.add_argument("--output", default="config", choices=["config", "raw", "proba", "leaf"],
                    help="output kind: the config's (default), raw margins, predict_proba, or "
                         "leaf indices (rows x trees int32)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3)

    dist = Dist()
    cfg = synth.CONFIGS[args.config]
    if args.scaling is None:
        args.scaling = default_scaling(cfg)
    if args.workload == "contrib":
        run_contrib(args, dist, cfg)
        dist.close()
        return
    if args.workload == "binned":
        run_binned(args, dist, cfg)
        dist.close()
        return
    text = synth.model_to_json(synth.make_model(cfg))

    if args.impl == "reference":
        line = run_reference(args, dist, cfg, text)
        if line is not None:
            print(json.dumps(line), flush=True)
        dist.close()
        return

    import torch

    from macboost_b200 import _core

    dev = dist.local_rank
    torch.cuda.set_device(dev)
    affinity = bind_near_gpu(dev) if dist.world > 1 else None
    rows = rows_per_rank(cfg, args, dist.world)
    row_start = dist.rank * rows
    kind = OUTPUT_KIND[cfg.output] if args.output == "config" else \
        {"raw": 1, "proba": 2, "leaf": 3}[args.output]
    odt = np.int32 if kind == 3 else np.float32
    h = _core.load_json(text)
    _core.prepare(h, [dev])
    desc = json.loads(_core.describe(h))
    S = desc["slots"]
    ocols = _core.output_cols(h, kind)

    # inputs: seeded, this rank's shard, feature-major in page-locked memory
    Xh = _core.pinned_empty((cfg.features, rows))
    synth.make_data(cfg, rows=rows, row_start=row_start, layout="feature", out=Xh)
    outh = _core.pinned_empty((rows, ocols), dtype=odt)
    xd = torch.from_numpy(np.asarray(Xh)).to(f"cuda:{dev}")
    outd = torch.empty((rows, ocols), dtype=torch.int32 if kind == 3 else torch.float32,
                       device=f"cuda:{dev}")
    stream = torch.cuda.current_stream(dev)

    def step():
        _core.predict_device(h, dev, xd.data_ptr(), rows, cfg.features, rows, outd.data_ptr(),
                             kind=kind, stream=stream.cuda_stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    _core.check_device(h, dev)

    clocks = ClockSampler(dev)
    clocks.start()
    dist.barrier()
    torch.cuda.synchronize(dev)
    launches0 = _core.kernel_launches()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    # sample while the queued steps run (a blocking synchronize can keep the
    # sampler thread from running); the device timing is unaffected
    clocks.sample()
    while not ev1.query():
        clocks.sample()
        time.sleep(0.001)
    torch.cuda.synchronize(dev)
    dist.barrier()
    launches = _core.kernel_launches() - launches0
    ms_local = ev0.elapsed_time(ev1)
    _core.check_device(h, dev)
    clk = clocks.stop()
    ms = dist.max(ms_local)
    per_step_s = ms / 1e3 / args.steps
    units = rows * cfg.trees * dist.world
    value = units / per_step_s

    # the step's output, and the raw margins of the same rows (one more
    # launch, after the timed region), for the parity check of the CPU leg
    out_gpu = outd.cpu().numpy()
    raw_gpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        K = cfg.classes
        rawd = torch.empty((rows, K), dtype=torch.float32, device=f"cuda:{dev}")
        _core.predict_device(h, dev, xd.data_ptr(), rows, cfg.features, rows, rawd.data_ptr(),
                             kind=1, stream=stream.cuda_stream)
        torch.cuda.synchronize(dev)
        _core.check_device(h, dev)
        raw_gpu = rawd.cpu().numpy()
        del rawd

    # end to end through the reference-facing C ABI with host buffers
    e2e_s = None
    ceiling = None
    if args.e2e_steps > 0:
        _core.predict_ex(h, np.asarray(Xh), kind=kind, layout="feature", devices=[dev], out=outh)
        dist.barrier()
        e2e_times = []
        for _ in range(args.e2e_steps):
            dist.barrier()
            t0 = time.perf_counter()
            _core.predict_ex(h, np.asarray(Xh), kind=kind, layout="feature", devices=[dev],
                             out=outh)
            e2e_times.append(time.perf_counter() - t0)
        e2e_s = dist.max(sum(e2e_times) / len(e2e_times))
        ceiling = copy_ceiling(dist, dev, stream, rows * S * 4, rows * ocols * 4, e2e_s)

    peak, peak_src = measured_peak_hbm()
    alg_bytes = rows * 4 * (S + ocols)
    # this rank's kernel: one launch per step, timed on its launching stream
    achieved = alg_bytes / (ms_local / 1e3 / args.steps) / 1e9
    tr = traffic_lookup(cfg.name if args.output == "config" else f"{cfg.name}_{args.output}")
    line = {
        "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms / args.steps,
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f32", "data": "synthetic (seeded model and rows; no dataset)",
        "config": dict(config_block(cfg, rows, args),
                       **({} if args.output == "config" else {"output": args.output})),
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                     "frac": achieved / peak, "peak_source": peak_src,
                     "traffic": (tr["bytes_per_row"] * rows) if tr else None,
                     "algorithmic_bytes_per_launch": alg_bytes,
                     "note": "algorithmic bytes = rows*4*(used features + output columns); "
                             "the tree walk is bound by shared-memory wavefronts, not HBM"},
        "e2e": None if e2e_s is None else {
            "value": units / e2e_s, "unit": UNIT,
            "h2d_bytes_per_step": rows * S * 4, "d2h_bytes_per_step": rows * ocols * 4,
            "ms_per_step": e2e_s * 1e3,
            "frac_of_copy_ceiling": None if ceiling is None else ceiling["copy_ms"] / (e2e_s * 1e3)},
        "e2e_copy_ceiling": ceiling,
        "gpu_launches": int(launches),
        "clocks": clk,
        "layout": desc,
    }
    if affinity:
        line["host_affinity"] = affinity
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        base, raw_o, om = cpu_baseline(cfg, text, np.asarray(Xh))
        line["cpu_baseline"] = base
        from oracle import oracle as O
        leaf_o = None
        if kind == 3:
            n = raw_o.shape[0]
            _, leaf_o = O.predict_raw(om, np.ascontiguousarray(np.asarray(Xh)[:, :n]),
                                      layout="feature", want_leaf=True)
        line["parity"] = parity_check(O, om, raw_o, raw_gpu, out_gpu, kind, leaf_o)
        ref = reference_pymodel(cfg, text, np.asarray(Xh))
        if ref is not None:
            line["cpu_baseline_reference"] = ref
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    del xd, outd
    dist.close()


def copy_ceiling(dist, dev, stream, h2d_bytes, d2h_bytes, e2e_s):
    """Plain page-locked copies of an e2e step's bytes, every rank at once:
    H2D of the input and D2H of the output, timed with CUDA events on the
    bench stream (best of 3 after one warm-up, max over ranks)."""
    import torch
    hin = torch.empty(h2d_bytes // 4, dtype=torch.float32, pin_memory=True)
    din = torch.empty(h2d_bytes // 4, dtype=torch.float32, device=f"cuda:{dev}")
    hout = torch.empty(max(d2h_bytes // 4, 1), dtype=torch.float32, pin_memory=True)
    dout = torch.empty(max(d2h_bytes // 4, 1), dtype=torch.float32, device=f"cuda:{dev}")

    def timed(fn):
        best = None
        for i in range(4):
            dist.barrier()
            torch.cuda.synchronize(dev)
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            fn()
            e1.record(stream)
            e1.synchronize()
            if i:
                t = e0.elapsed_time(e1)
                best = t if best is None else min(best, t)
        return dist.max(best)

    h2d_ms = timed(lambda: din.copy_(hin, non_blocking=True))
    d2h_ms = timed(lambda: hout.copy_(dout, non_blocking=True))
    del hin, din, hout, dout
    return {"h2d_gbs": h2d_bytes / h2d_ms / 1e6, "d2h_gbs": d2h_bytes / d2h_ms / 1e6,
            "copy_ms": h2d_ms + d2h_ms, "ranks_copying_at_once": dist.world,
            "note": "plain cudaMemcpyAsync (torch copy_) of the step's input and output "
                    "bytes from/to page-locked memory, all ranks at once, max over ranks; "
                    "e2e.frac_of_copy_ceiling = copy_ms / e2e ms_per_step"}


def _time_steps(step, steps, warmup, stream, dist, clocks=None):
    """Device time of `steps` launches on `stream` (ms, max over ranks)."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    if clocks:
        clocks.start()
    dist.barrier()
    torch.cuda.synchronize()
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    ev0.record(stream)
    for _ in range(steps):
        step()
    ev1.record(stream)
    if clocks:
        # sample while the queued launches run (a blocking synchronize can keep
        # the sampler thread from running); the device timing is unaffected
        clocks.sample()
        while not ev1.query():
            clocks.sample()
            time.sleep(0.001)
    torch.cuda.synchronize()
    dist.barrier()
    ms_local = ev0.elapsed_time(ev1)
    clk = clocks.stop() if clocks else None
    return dist.max(ms_local), ms_local, clk


CONTRIB_ROWS = {"cfg1": 500_000, "cfg2": 1_000_000, "cfg3": 500_000, "cfg4": 100_000,
                "cfg5": 100_000}


def run_contrib(args, dist, cfg):
    """--workload contrib: TreeSHAP contributions (macboost_predict_contrib_device) on
    the config's model with node covers from 20,000 routed rows, device-resident
    feature-major input; e2e through macboost_predict_contrib_ex on pinned buffers."""
    import torch

    from macboost_b200 import _core
    dev = dist.local_rank
    torch.cuda.set_device(dev)
    rows = args.rows or CONTRIB_ROWS[cfg.name]
    trees = args.trees or cfg.trees
    model = synth.make_model(cfg, trees=trees)
    synth.add_covers(model, synth.make_data(cfg, rows=20_000, seed=cfg.data_seed + 7,
                                            layout="row"))
    text = synth.model_to_json(model)
    h = _core.load_json(text)
    _core.prepare(h, [dev])
    F, K = cfg.features, cfg.classes
    W = K * (F + 1)
    Xh = _core.pinned_empty((F, rows))
    synth.make_data(cfg, rows=rows, row_start=dist.rank * rows, layout="feature", out=Xh)
    xd = torch.from_numpy(np.asarray(Xh)).to(f"cuda:{dev}")
    outd = torch.empty((rows, W), dtype=torch.float32, device=f"cuda:{dev}")
    stream = torch.cuda.current_stream(dev)

    def step():
        _core.predict_contrib_device(h, dev, xd.data_ptr(), rows, F, rows, outd.data_ptr(),
                                     stream=stream.cuda_stream)

    launches0 = _core.kernel_launches()
    ms, ms_local, clk = _time_steps(step, args.steps, args.warmup, stream, dist,
                                    ClockSampler(dev))
    launches = _core.kernel_launches() - launches0 - args.warmup
    _core.check_device(h, dev)
    per_step = ms / 1e3 / args.steps
    units = rows * trees * dist.world
    e2e = None
    if args.e2e_steps > 0:
        outh = _core.pinned_empty((rows, W))
        ts = []
        for _ in range(args.e2e_steps + 1):
            dist.barrier()
            t0 = time.perf_counter()
            _core.predict_contrib_ex(h, np.asarray(Xh), layout="feature", devices=[dev])
            ts.append(time.perf_counter() - t0)
        e2e_s = dist.max(sum(ts[1:]) / len(ts[1:]))
        e2e = {"value": units / e2e_s, "unit": UNIT, "h2d_bytes_per_step": rows * F * 4,
               "d2h_bytes_per_step": rows * W * 4}
        del outh
    peak, peak_src = measured_peak_hbm()
    alg = rows * 4 * (F + W)
    line = {
        "metric": "TreeSHAP contributions rows·trees/s", "value": units / per_step,
        "unit": UNIT, "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded model and rows)",
        "config": {"workload": f"contrib on {cfg.name}: {rows} rows x {trees} trees, "
                               f"covers from 20,000 routed rows",
                   "rows_per_gpu": rows, "features": F, "trees": trees, "classes": K,
                   "output": "rows x K x (F+1) float32",
                   "l2": "inputs and outputs larger than L2" if alg > (126 << 20)
                         else "output written once per step"},
        "roofline": {"bound": "hbm", "achieved": alg / (ms_local / 1e3 / args.steps) / 1e9,
                     "peak": peak, "unit": "GB/s", "peak_source": peak_src,
                     "frac": alg / (ms_local / 1e3 / args.steps) / 1e9 / peak,
                     "traffic": None, "algorithmic_bytes_per_launch": alg,
                     "note": "float64 path arithmetic bound (latency and occupancy), "
                             "not HBM: bytes = input values + contribution outputs"},
        "e2e": e2e, "gpu_launches": int(launches), "clocks": clk,
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        from oracle import oracle as O
        O.build()
        om = O.model_from_dict(json.loads(text))
        n = 256 if trees * cfg.features <= 20_000 else 64
        Xs = synth.make_data(cfg, rows=n, seed=cfg.data_seed + 99, layout="row")
        t0 = time.perf_counter()
        O.predict_contrib(om, Xs)
        dt = time.perf_counter() - t0
        line["cpu_baseline"] = {
            "value": n * trees / dt, "unit": UNIT, "cores": os.cpu_count() or 1, "kind": "port",
            "sample": f"{n} rows x {trees} trees, {dt:.2f} s (oracle/mbshap.c, restatement "
                      f"of SHAP.swift's recursive CPU TreeSHAP)"}
    if dist.rank == 0:
        print(json.dumps(line), flush=True)
    del xd, outd


def run_binned(args, dist, cfg):
    """--workload binned: per step, one depth-6 tree in split form walked over the
    config's rows in the trainer's tiled bin layout (predict_tree_binned + its leaf
    indices, device memory), as a trainer evaluates each new tree; the line also
    times bin_data on the same rows."""
    import ctypes

    import torch

    from macboost_b200 import _core
    dev = dist.local_rank
    torch.cuda.set_device(dev)
    rows = (args.rows or cfg.rows) // 2 * 2
    F, nb, depth = cfg.features, 256, 6
    groups = (F + 7) // 8
    rng = np.random.default_rng(cfg.model_seed + 11)
    n_nodes = (1 << (depth + 1)) - 1
    feat = np.full(n_nodes, -1, np.int32)
    feat[: (1 << depth) - 1] = rng.integers(0, F, (1 << depth) - 1)
    sbin = rng.integers(0, nb - 2, n_nodes).astype(np.uint32)
    flags = rng.integers(0, 2, n_nodes).astype(np.uint32)
    leaf = rng.standard_normal(n_nodes).astype(np.float32)
    g = torch.Generator(device=f"cuda:{dev}").manual_seed(cfg.data_seed)
    bins = torch.randint(0, nb, (groups * 8 * rows,), dtype=torch.uint8, device=f"cuda:{dev}",
                         generator=g)
    d = {k: torch.from_numpy(v).to(f"cuda:{dev}") for k, v in
         (("off", np.array([0, n_nodes], np.int64)), ("feat", feat), ("sbin", sbin.view(np.int32)),
          ("flags", flags.view(np.int32)), ("mask", np.zeros(n_nodes * 8, np.int32)),
          ("leaf", leaf))}
    preds = torch.zeros(rows, dtype=torch.float32, device=f"cuda:{dev}")
    leafidx = torch.empty(rows, dtype=torch.int32, device=f"cuda:{dev}")
    status = torch.zeros(1, dtype=torch.int32, device=f"cuda:{dev}")
    stream = torch.cuda.current_stream(dev)
    lib = _core._lib
    P, I32, I64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
    fn = lib.macboost_predict_tree_binned_device
    fn.restype = I32
    fn.argtypes = [P, I64, I64, I32, I32, P, P, P, P, P, P, I32, I32, I32, P, P, P, P,
                   ctypes.POINTER(ctypes.c_char_p)]
    err = ctypes.c_char_p()

    def step():
        if fn(bins.data_ptr(), rows, F, nb, 1, d["off"].data_ptr(), d["feat"].data_ptr(),
              d["sbin"].data_ptr(), d["flags"].data_ptr(), d["mask"].data_ptr(),
              d["leaf"].data_ptr(), depth, 1, dev, preds.data_ptr(), leafidx.data_ptr(),
              status.data_ptr(), stream.cuda_stream, ctypes.byref(err)) != 0:
            raise RuntimeError(err.value)

    launches0 = _core.kernel_launches()
    ms, ms_local, clk = _time_steps(step, args.steps, args.warmup, stream, dist,
                                    ClockSampler(dev))
    launches = _core.kernel_launches() - launches0 - args.warmup
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    # bin_data on the config's rows (device-resident, feature-major)
    x = torch.from_numpy(synth.make_data(cfg, rows=rows, layout="feature")).to(f"cuda:{dev}")
    edges = torch.from_numpy(np.sort(rng.standard_normal((F, nb - 2)), axis=1)
                             .astype(np.float32)).to(f"cuda:{dev}")
    cat = torch.zeros(F, dtype=torch.uint8, device=f"cuda:{dev}")
    fb = lib.macboost_bin_data_device
    fb.restype = I32
    fb.argtypes = [P, I64, I64, I64, I32, P, I32, P, I32, P, P, ctypes.POINTER(ctypes.c_char_p)]

    def bstep():
        if fb(x.data_ptr(), rows, F, rows, 0, edges.data_ptr(), nb, cat.data_ptr(), dev,
              bins.data_ptr(), stream.cuda_stream, ctypes.byref(err)) != 0:
            raise RuntimeError(err.value)

    bms, bms_local, _ = _time_steps(bstep, args.steps, args.warmup, stream, dist)
    peak, peak_src = measured_peak_hbm()
    per_row = groups * 8 + 4 + 4 + 4          # tile words + preds read/write + leaf index
    t_step = ms_local / 1e3 / args.steps
    line = {
        "metric": "binned tree walk rows·trees/s", "value": rows * dist.world / (ms / 1e3 / args.steps),
        "unit": UNIT, "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": args.scaling,
        "vs_baseline": None, "dtype": "u8", "data": "synthetic (random bins and tree)",
        "config": {"workload": f"binned on {cfg.name}: {rows} rows x {F} features "
                               f"({groups} tiles of 8), one depth-6 tree per step, "
                               f"predict_tree_binned + assign_leaves",
                   "rows_per_gpu": rows, "features": F, "trees": 1, "num_bins": nb,
                   "l2": "bin matrix larger than L2 (streamed once per step)"},
        "roofline": {"bound": "hbm", "achieved": rows * per_row / t_step / 1e9, "peak": peak,
                     "unit": "GB/s", "peak_source": peak_src,
                     "frac": rows * per_row / t_step / 1e9 / peak, "traffic": None,
                     "algorithmic_bytes_per_launch": rows * per_row,
                     "note": "bytes = the rows' tile words + preds read/write + leaf index"},
        "bin_data": {"ms_per_step": bms / args.steps,
                     "achieved_gbs": rows * F * 5 / (bms_local / 1e3 / args.steps) / 1e9,
                     "note": "reads F x 4 B values, writes F bin bytes per row"},
        "e2e": None, "gpu_launches": int(launches), "clocks": clk,
    }
    if dist.rank == 0:
        print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
