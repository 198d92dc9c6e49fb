#!/usr/bin/env python
"""Benchmark of the B200 grammar-conditioned LM head.

Headline workload (one GPU): batch-1 row-sparse (direct-bitmask) projection at
V=248,320, H=2,048, fp16, W ~ N(0, 0.02), h ~ N(0, 1), 1% of the vocabulary
legal (uniform), a fresh seeded mask every step. One step = one call of the
hot path: full -inf-filled logits [V] plus the fused greedy top-1.

  value      legal-row GB/s = legal W bytes (k * H * 2) per step / device time
             per step, summed over ranks' work, timed with CUDA events;
  e2e        the same metric through the C-ABI call with host buffers: the
             step's mask and hidden state copied from pinned host memory to
             the device (gsp_copy_bytes), the top-1 record stored by the
             kernel into pinned host memory, all inside the timed region;
  roofline   the row-sparse kernel's achieved legal-row bandwidth against the
             measured HBM copy bandwidth;
  sweep      every density of the GEMV workload, uniform and clustered;
  cpu_baseline  the oracle's CPU restatement of the same step on host cores.

Timing (one GPU): the K timed steps are captured in one CUDA graph and timed
with CUDA events around its replay, so host launch overhead and per-step event
overhead are excluded. Inputs are larger than L2: step i reads weight copy
i % 32 (32 copies of the 1 GB head) and mask i % 64, so no step finds its legal
rows in L2. A second, conservative figure ("cold") times every step eagerly
with its own events after a 256 MiB L2-flushing write. With --gpus N (torchrun,
one process per GPU) the head is vocabulary-parallel: each rank streams the
legal rows of its V/N shard and the projection kernel's last CTA merges the
per-request top-1 with the other ranks over peer memory (NVLink), inside the
same launch.

`--impl reference` times the reference's CPU algorithm for the same step (the
oracle port, all host threads) and prints its own line.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(REPO, "grammar-sparse-projection_b200"))
sys.path.insert(0, REPO)

import numpy as np  # noqa: E402
import torch  # noqa: E402

METRIC = "LM-head µs/step & legal-row HBM GB/s at V=248320 H=2048 fp16, batch 1-32"
UNIT = "GB/s"
VOCAB, HIDDEN = 248320, 2048
DENSITIES = (0.0005, 0.005, 0.01, 0.10, 0.50, 1.0)
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=1000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("ours", "reference"), default="ours")
    ap.add_argument("--density", type=float, default=0.01)
    ap.add_argument("--pattern", choices=("uniform", "clustered"), default="uniform")
    ap.add_argument("--masks", type=int, default=64, help="distinct seeded masks cycled through")
    ap.add_argument("--copies", type=int, default=32, help="weight copies cycled through (one GPU)")
    ap.add_argument("--sweep-steps", type=int, default=100)
    ap.add_argument("--no-sweep", action="store_true")
    ap.add_argument("--no-vp", action="store_true", help="skip the vocabulary-parallel head section")
    ap.add_argument("--only", choices=("batched", "mixed", "vp", "sampler", "graphed", "groups", "reference-triton",
                                       "kernel"),
                    default=None,
                    help="run one extra section alone (small; for profiling)")
    ap.add_argument("--batch", type=int, default=32, help="batch of --only batched")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--ref-out", default=None, help="(reference-triton child) file for its step-0 logits")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def make_masks(n: int, density: float, pattern: str, seed: int) -> np.ndarray:
    from gsp import workloads as wl
    rng = np.random.default_rng(seed)
    k = int(round(density * VOCAB))
    return np.concatenate([wl.make_batch_mask(rng, 1, VOCAB, [k], clustered=(pattern == "clustered"),
                                             max_runs=64) for _ in range(n)])


def legal_counts(masks: np.ndarray) -> np.ndarray:
    from gsp import workloads as wl
    return wl.unpack_bitmask(masks, VOCAB).sum(axis=1)


def read_peaks():
    path = os.path.join(REPO, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            peaks = json.load(f)
        return float(peaks["hbm_gbs"]), "measured (MEASURED_PEAKS.json hbm_gbs)"
    except (OSError, KeyError, ValueError):
        return FALLBACK_HBM_GBS, "fallback"


TRAFFIC_CSV = os.path.join("profiles", "row_sparse_staged_b1_1pct_dram.csv")


def read_traffic_csv(kernel_substr: str = "row_sparse_staged_kernel", path: str = TRAFFIC_CSV):
    """Per-launch DRAM traffic (dram__bytes_read.sum + dram__bytes_write.sum,
    mean over the captured launches of `kernel_substr`) from an ncu CSV
    (`ncu --csv --print-units base --metrics ...`) committed under profiles/.
    Returns (bytes or None, source description). Not measured by this run:
    the capture's command is in the CSV's companion summary."""
    import csv
    full = os.path.join(REPO, path)
    try:
        rows = list(csv.DictReader(open(full)))
    except OSError:
        return None, f"no ncu capture at {path}"
    per_launch = {}
    for r in rows:
        if kernel_substr not in r.get("Kernel Name", ""):
            continue
        if r.get("Metric Name") in ("dram__bytes_read.sum", "dram__bytes_write.sum"):
            unit = (r.get("Metric Unit") or "byte").strip()
            scale = {"byte": 1, "Kbyte": 1e3, "Mbyte": 1e6, "Gbyte": 1e9}.get(unit, 1)
            per_launch[r["ID"]] = per_launch.get(r["ID"], 0.0) + float(r["Metric Value"].replace(",", "")) * scale
    if not per_launch:
        return None, f"no {kernel_substr} launch in {path}"
    return (statistics.mean(per_launch.values()),
            f"ncu capture committed at {path} ({len(per_launch)} launches), not this run")


def exact_check(hidden, weight, mask, logits, top_index, *, rtol=2e-3, atol=2e-3, chunk_rows=32768):
    """Checks one timed step's outputs on the device against exact float64
    products (plain torch): legal support bit-exact (-inf on every illegal
    token), each legal logit within atol + max(rtol |x|, half an output ulp),
    the fused top-1 equal to argmax of the logits and within the near-tie
    window of the exact maximum. Returns a small dict for the JSON line."""
    batch, vocab = logits.shape
    v = torch.arange(vocab, device=logits.device)
    legal = ((mask.reshape(batch, -1)[:, v >> 5] >> (v & 31)) & 1).bool()
    lg = logits.double()
    support = bool(torch.equal(torch.isfinite(lg), legal)) and bool(torch.isneginf(lg[~legal]).all())
    h64 = hidden.double()
    exact = torch.empty(batch, vocab, dtype=torch.float64, device=logits.device)
    for r0 in range(0, vocab, chunk_rows):
        r1 = min(vocab, r0 + chunk_rows)
        exact[:, r0:r1] = h64 @ weight[r0:r1].double().T
    exact.masked_fill_(~legal, float("-inf"))
    mant = {torch.float16: 10, torch.bfloat16: 7}.get(logits.dtype, 23)
    fin = legal
    ax = exact[fin].abs().clamp_min(2.0 ** -14)
    half_ulp = 0.5 * torch.exp2(torch.floor(torch.log2(ax)) - mant)
    diff = (lg[fin] - exact[fin]).abs()
    values = bool((diff <= atol + torch.maximum(rtol * exact[fin].abs(), half_ulp)).all()) if fin.any() else True
    top_ok = bool(torch.equal(top_index.reshape(-1), logits.argmax(-1)))
    best = exact.max(dim=-1).values
    picked = exact.gather(1, top_index.reshape(-1, 1))[:, 0]
    window = atol + torch.maximum(rtol * best.abs(), torch.exp2(torch.floor(torch.log2(best.abs().clamp_min(2.0 ** -14))) - mant))
    has = torch.isfinite(best)
    top_ok &= bool(((best - picked <= window) | ~has).all())
    return {"support": support, "values": values, "top1": top_ok,
            "max_abs_err": float(diff.max()) if fin.any() else 0.0,
            "method": "float64 torch products on the device, the tolerance of the parity tests"}


# ---------------------------------------------------------------------------
# clocks during the timed region (NVML polling thread; read-only)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80, "display_clock_setting": 0x100,
    }

    def __init__(self, device_index: int, period_s: float = 0.002):
        self.samples, self.reasons, self.max_mhz = [], set(), None
        self._stop = threading.Event()
        self._period = period_s
        self._handle = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(device_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._handle = None

    def _run(self):
        nv = self._nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self._handle, nv.NVML_CLOCK_SM))
                mask = nv.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                for name, bit in self.REASONS.items():
                    if mask & bit:
                        self.reasons.add(name)
            except Exception:
                break
            time.sleep(self._period)

    def __enter__(self):
        if self._handle is not None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._handle is not None:
            self._stop.set()
            self._t.join()

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": sorted(self.reasons),
                    "samples": 0, "source": "nvml unavailable"}
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": sorted(self.reasons - {"gpu_idle"}), "samples": len(self.samples),
                "source": "nvml"}


# ---------------------------------------------------------------------------
# CPU side: baseline and reference arm
# ---------------------------------------------------------------------------
def cpu_threads() -> int:
    try:
        from threadpoolctl import threadpool_info
        info = [i for i in threadpool_info() if i.get("user_api") == "blas"]
        if info:
            return int(max(i["num_threads"] for i in info))
    except Exception:
        pass
    return os.cpu_count() or 1


def time_cpu_steps(weight_cpu: np.ndarray, hidden_cpu: np.ndarray, masks: np.ndarray, steps: int | None,
                   seconds: float | None):
    """Times oracle.cpu_row_sparse_step over cycling masks; returns (GB/s, µs/step, steps)."""
    from oracle import gsp_oracle as O
    counts = legal_counts(masks)
    done, legal_bytes, t0 = 0, 0, time.perf_counter()
    while True:
        m = masks[done % len(masks)][None]
        O.cpu_row_sparse_step(hidden_cpu, weight_cpu, m, VOCAB)
        legal_bytes += int(counts[done % len(masks)]) * HIDDEN * 2
        done += 1
        el = time.perf_counter() - t0
        if steps is not None and done >= steps:
            break
        if seconds is not None and el >= seconds and done >= 3:
            break
    el = time.perf_counter() - t0
    return legal_bytes / el / 1e9, el / done * 1e6, done


REF_DIR = os.path.join(REPO, "baseline", "_ref")


def reference_runtime():
    """The reference's own gsp/runtime.py from the unmodified copy under
    baseline/_ref (baseline/install_reference.py), loaded under its own module
    name; None when the copy is absent."""
    import importlib.util
    path = os.path.join(REF_DIR, "gsp", "runtime.py")
    if not os.path.exists(path):
        return None
    spec = importlib.util.spec_from_file_location("gsp_reference_runtime", path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def time_cpu_reference_sparse(weight_cpu: np.ndarray, hidden_cpu: np.ndarray, masks: np.ndarray,
                              steps: int | None, seconds: float | None):
    """The reference's own CPU path for the step (gsp/runtime.py:16-51,
    constrained_projection on CPU tensors; sparse-gather below 30% legal):
    the mask row's legal ids, the projection of those rows, the -inf-filled
    vocabulary row and its argmax. Returns (GB/s, us/step, steps) or None."""
    from gsp import workloads as wl
    ref = reference_runtime()
    if ref is None:
        return None
    w = torch.from_numpy(weight_cpu)
    h = torch.from_numpy(hidden_cpu)
    counts = legal_counts(masks)
    done, legal_bytes, t0 = 0, 0, time.perf_counter()
    while True:
        m = masks[done % len(masks)][None]
        ids = torch.from_numpy(np.flatnonzero(wl.unpack_bitmask(m, VOCAB)[0]))
        res = ref.constrained_projection(h, w, ids)
        full = torch.full((VOCAB,), float("-inf"), dtype=w.dtype)
        full[res.token_ids] = res.logits[0]
        int(full.argmax())
        legal_bytes += int(counts[done % len(masks)]) * HIDDEN * 2
        done += 1
        el = time.perf_counter() - t0
        if steps is not None and done >= steps:
            break
        if seconds is not None and el >= seconds and done >= 3:
            break
    el = time.perf_counter() - t0
    return legal_bytes / el / 1e9, el / done * 1e6, done


def time_cpu_reference_dense(weight_cpu: np.ndarray, hidden_cpu: np.ndarray, masks: np.ndarray, seconds: float):
    """The reference's dense route on the host (gsp/triton_runtime.py:302-307
    with xgrammar's CPU mask kernel): F.linear over every row, the mask applied
    in place, argmax. Returns (GB/s of legal rows, us/step, steps) or None."""
    try:
        import torch.nn.functional as F
        import xgrammar as xgr
    except ImportError:
        return None
    w = torch.from_numpy(weight_cpu)
    h = torch.from_numpy(hidden_cpu)
    counts = legal_counts(masks)
    done, legal_bytes, t0 = 0, 0, time.perf_counter()
    while True:
        m = torch.from_numpy(masks[done % len(masks)][None])
        lg = F.linear(h, w)
        xgr.apply_token_bitmask_inplace(lg, m, vocab_size=VOCAB, backend="cpu")
        int(lg.argmax())
        legal_bytes += int(counts[done % len(masks)]) * HIDDEN * 2
        done += 1
        el = time.perf_counter() - t0
        if el >= seconds and done >= 2:
            break
    return legal_bytes / el / 1e9, el / done * 1e6, done


def cpu_baselines(weight_cpu, hidden_cpu, masks, seconds: float, density: float, pattern: str):
    """Every CPU figure for the headline step, on this host's cores: the
    reference's own sparse path (the baseline when its copy is present), its
    dense route with xgrammar's CPU mask, and the oracle's restatement."""
    torch.set_num_threads(os.cpu_count() or 1)
    what = f"batch 1, V={VOCAB}, H={HIDDEN} fp16, {density:.2%} {pattern}"
    out = {}
    r = time_cpu_reference_sparse(weight_cpu, hidden_cpu, masks, steps=None, seconds=seconds)
    if r is not None:
        out["reference_sparse"] = {"value": r[0], "unit": UNIT, "us_per_step": r[1], "cores": cpu_threads(),
                                   "kind": "reference",
                                   "sample": (f"{r[2]} steps ({r[1]:.0f} us/step) of the reference's own "
                                              f"constrained_projection on CPU tensors (unmodified copy under "
                                              f"baseline/_ref) + -inf row + argmax, {what}, bounded to "
                                              f"{seconds:.0f} s")}
    d = time_cpu_reference_dense(weight_cpu, hidden_cpu, masks, seconds=min(seconds, 5.0))
    if d is not None:
        out["reference_dense"] = {"value": d[0], "unit": UNIT, "us_per_step": d[1], "cores": cpu_threads(),
                                  "kind": "reference",
                                  "sample": (f"{d[2]} steps of F.linear + xgrammar apply_token_bitmask_inplace("
                                             f"backend='cpu') + argmax, {what}")}
    gbs, us, n = time_cpu_steps(weight_cpu, hidden_cpu, masks, steps=None, seconds=seconds)
    out["port"] = {"value": gbs, "unit": UNIT, "us_per_step": us, "cores": cpu_threads(), "kind": "port",
                   "sample": f"{n} steps ({us:.0f} us/step) of the oracle's restatement, {what}"}
    head = dict(out.get("reference_sparse") or out["port"])
    head["others"] = {k: v for k, v in out.items() if v is not None and v.get("sample") != head.get("sample")}
    return head


def host_weight(seed: int) -> tuple[np.ndarray, np.ndarray]:
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(VOCAB, HIDDEN, generator=g) * 0.02).half().numpy()
    h = torch.randn(1, HIDDEN, generator=g).half().numpy()
    return w, h


def run_reference_arm(args):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return 0
    torch.set_num_threads(os.cpu_count() or 1)
    masks = make_masks(args.masks, args.density, args.pattern, seed=100)
    w, h = host_weight(1234)
    what = f"at V={VOCAB}, H={HIDDEN} fp16, {args.density:.2%} {args.pattern}"
    kind = "reference"
    if time_cpu_reference_sparse(w, h, masks, steps=max(args.warmup, 1), seconds=None) is not None:
        gbs, us, n = time_cpu_reference_sparse(w, h, masks, steps=args.steps, seconds=None)
        sample = (f"{n} steps of the reference's own CPU path (gsp.runtime.constrained_projection on CPU "
                  f"tensors from the unmodified copy under baseline/_ref, then the -inf-filled row and its "
                  f"argmax) {what}")
    else:
        kind = "port"
        time_cpu_steps(w, h, masks, steps=max(args.warmup, 1), seconds=None)
        gbs, us, n = time_cpu_steps(w, h, masks, steps=args.steps, seconds=None)
        sample = (f"{n} steps of the oracle's restatement of the batch-1 row-sparse step (mask decode, "
                  f"legal-row gather, fp32 dots, -inf fill, argmax) {what}; the reference copy under "
                  f"baseline/_ref is absent")
    line = {
        "metric": METRIC, "value": gbs, "unit": UNIT, "impl": "reference", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": us / 1e3, "us_per_step": us,
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f16",
        "data": "synthetic",
        "config": workload_config(args),
        "cpu_baseline": {"value": gbs, "unit": UNIT, "cores": cpu_threads(), "kind": kind, "sample": sample},
        "e2e": {"value": gbs, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)
    return 0


def run_kernel_only(args):
    """The headline step alone, eagerly, --warmup + --steps times over
    --copies weight copies and --masks masks: the command the committed ncu
    captures of the row-sparse kernel run (a few GB on the device)."""
    from gsp import _native
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1234)
    weights = [(torch.randn(VOCAB, HIDDEN, device=dev, generator=g) * 0.02).half() for _ in range(args.copies)]
    hidden = torch.randn(1, HIDDEN, device=dev, generator=torch.Generator(device=dev).manual_seed(99)).half()
    masks_np = make_masks(args.masks, args.density, args.pattern, seed=100)
    masks = torch.from_numpy(masks_np).to(dev)
    logits = torch.empty(1, VOCAB, device=dev, dtype=torch.float16)
    tv = torch.empty(1, device=dev)
    ti = torch.empty(1, device=dev, dtype=torch.int64)
    for i in range(args.warmup + args.steps):
        _native.row_sparse(hidden, weights[i % len(weights)], masks[i % len(masks)][None], logits=logits,
                           top_value=tv, top_index=ti)
    torch.cuda.synchronize()
    counts = legal_counts(masks_np)
    print(json.dumps({"only": "kernel", "launches": args.warmup + args.steps,
                      "legal_bytes_per_launch_mean": float(np.mean(counts)) * HIDDEN * 2}), flush=True)
    return 0


def run_reference_triton(args):
    """Child process of reference_triton_section: the reference's own Triton
    kernels (gsp/triton_runtime.py:15-125, 147-258 of the unmodified copy
    under baseline/_ref) through its public wrappers, on the headline workload
    (batch 1, the same seeded weights, hidden state and masks) and the batched
    block-GEMM workload; CUDA-graph timed like this library's routes. Prints
    one JSON object; saves its step-0 logits (int16 view) to --ref-out."""
    import importlib.util
    try:
        sys.path.insert(0, REF_DIR)
        import gsp.triton_runtime as ref  # the reference's package, first on the path
        if not os.path.abspath(ref.__file__).startswith(os.path.abspath(REF_DIR)):
            raise ImportError(f"gsp resolved to {ref.__file__}, not the copy under baseline/_ref")
    except Exception as exc:
        print(json.dumps({"unavailable": f"{type(exc).__name__}: {exc}"}), flush=True)
        return 0
    spec = importlib.util.spec_from_file_location(
        "gsp_b200_workloads", os.path.join(REPO, "grammar-sparse-projection_b200", "gsp", "workloads.py"))
    wl = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(wl)
    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    g = torch.Generator(device=dev).manual_seed(1234)
    weights = [(torch.randn(VOCAB, HIDDEN, device=dev, generator=g) * 0.02).half() for _ in range(8)]
    hidden = torch.randn(1, HIDDEN, device=dev, generator=torch.Generator(device=dev).manual_seed(99)).half()
    rng = np.random.default_rng(100)
    k = int(round(args.density * VOCAB))
    masks_np = np.concatenate([wl.make_batch_mask(rng, 1, VOCAB, [k], clustered=(args.pattern == "clustered"),
                                                  max_runs=64) for _ in range(args.masks)])
    masks = torch.from_numpy(masks_np).to(dev)
    counts = wl.unpack_bitmask(masks_np, VOCAB).sum(axis=1)
    out = {"source": "unmodified reference copy under baseline/_ref, Triton " + __import__("triton").__version__}
    steps = 20
    try:
        t = graph_time_us(dev, steps, lambda i: ref.bitmask_sparse_logits(hidden, weights[i % 8], masks[i % len(masks)]))
        lb = float(sum(int(counts[i % len(masks)]) for i in range(steps))) * HIDDEN * 2
        out["batch1"] = {"us_per_step": t / steps, "legal_gbs": lb / (t * 1e-6) / 1e9,
                         "kernel": "_bitmask_sparse_lm_head_kernel via bitmask_sparse_logits"}
        lg = ref.bitmask_sparse_logits(hidden, weights[0], masks[0])
        torch.cuda.synchronize()
        if args.ref_out:
            np.save(args.ref_out, lg.view(torch.int16).cpu().numpy())
    except Exception as exc:
        out["batch1"] = {"unavailable": f"{type(exc).__name__}: {exc}"}
    batched = []
    for batch in (2, 4, 8, 16, 32):
        try:
            rng = np.random.default_rng(300 + batch)
            bm = [torch.from_numpy(wl.make_batch_mask(rng, batch, VOCAB, [1242] * batch, clustered=True,
                                                      max_runs=16)).to(dev) for _ in range(8)]
            hb = torch.randn(batch, HIDDEN, device=dev, generator=torch.Generator(device=dev).manual_seed(batch)).half()
            t = graph_time_us(dev, steps, lambda i: ref.bitmask_block_gemm_logits(hb, weights[i % 8], bm[i % 8]))
            batched.append({"batch": batch, "us_per_step": t / steps,
                            "kernel": "_bitmask_block_gemm_kernel via bitmask_block_gemm_logits"})
        except Exception as exc:
            batched.append({"batch": batch, "unavailable": f"{type(exc).__name__}: {exc}"})
    out["batched"] = batched
    print(json.dumps(out), flush=True)
    return 0


def reference_triton_section(dev, args, weights, hidden, masks, ours_us_per_step, batched):
    """The reference's Triton kernels on this GPU (child process: its package
    is also named gsp) beside this library's: timings, speed-ups, and the
    reference's step-0 logits against this library's on the same inputs."""
    import subprocess
    import tempfile
    from gsp import _native
    if not os.path.exists(os.path.join(REF_DIR, "gsp", "triton_runtime.py")):
        return {"unavailable": "no reference copy under baseline/_ref (baseline/install_reference.py)"}
    with tempfile.TemporaryDirectory() as tmp:
        ref_out = os.path.join(tmp, "ref_logits.npy")
        proc = subprocess.run([sys.executable, os.path.abspath(__file__), "--only", "reference-triton",
                               "--density", str(args.density), "--pattern", args.pattern, "--masks", str(args.masks),
                               "--ref-out", ref_out], capture_output=True, text=True, timeout=900)
        lines = [ln for ln in proc.stdout.splitlines() if ln.startswith("{")]
        if proc.returncode != 0 or not lines:
            return {"unavailable": f"child exited {proc.returncode}: {proc.stderr.strip()[-300:]}"}
        res = json.loads(lines[-1])
        if os.path.exists(ref_out):
            ref_bits = torch.from_numpy(np.load(ref_out)).to(dev)
            lg = torch.empty(1, VOCAB, device=dev, dtype=torch.float16)
            ti = torch.empty(1, device=dev, dtype=torch.int64)
            _native.row_sparse(hidden, weights[0], masks[0][None], logits=lg, top_index=ti)
            ref_lg = ref_bits.view(torch.float16).reshape(1, -1).float()
            ours = lg.float()
            fin = torch.isfinite(ref_lg)
            res["parity_vs_ours"] = {
                "support_equal": bool(torch.equal(fin, torch.isfinite(ours))),
                "max_abs_diff": float((ref_lg[fin] - ours[fin]).abs().max()) if fin.any() else 0.0,
                "argmax_equal": int(ref_lg.argmax()) == int(ti.item()),
                "what": "the reference kernel's step-0 logits vs this library's on the same W, h and mask"}
    b1 = res.get("batch1", {})
    if "us_per_step" in b1:
        b1["ours_us_per_step"] = ours_us_per_step
        b1["speedup_ours"] = b1["us_per_step"] / ours_us_per_step
    ours_block = {r["batch"]: r["us_per_step"] for r in (batched or [])}
    for r in res.get("batched", []):
        o = ours_block.get(r["batch"])
        if o and "us_per_step" in r:
            r["ours_block_us_per_step"] = o["block-sparse"]
            r["ours_best_us_per_step"] = min(v for k2, v in o.items() if k2 != "cublas+xgrammar" and v)
            r["speedup_ours_best"] = r["us_per_step"] / r["ours_best_us_per_step"]
    return res


def workload_config(args):
    return {"workload": "batch-1 row-sparse direct-bitmask LM-head GEMV", "vocab": VOCAB, "hidden": HIDDEN,
            "batch": 1, "density": args.density, "mask": f"{args.pattern}, fresh seeded mask per step",
            "weight": "fp16 N(0,0.02) row-major [V,H]", "outputs": "full logits [V] + fused top-1",
            "l2": ("inputs larger than L2: step i reads weight copy i % copies (each rank's shard of the "
                   "1 GB head) and mask i % masks"),
            "parallelism": (f"vocab-parallel x{args.gpus}: row shards of W, top-1 merged across ranks inside the "
                            "kernel over NVLink peer memory" if args.gpus > 1 else "single GPU")}


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
def main():
    args = parse_args()
    if args.impl == "reference":
        return run_reference_arm(args)
    if args.only == "reference-triton":
        return run_reference_triton(args)
    if args.only == "kernel":
        return run_kernel_only(args)
    if args.only:
        dev = torch.device("cuda", 0)
        torch.cuda.set_device(dev)
        peak, _ = read_peaks()
        if args.only == "batched":
            g = torch.Generator(device=dev).manual_seed(1234)
            weights = [(torch.randn(VOCAB, HIDDEN, device=dev, generator=g) * 0.02).half() for _ in range(2)]
            res = batched_section(dev, weights, peak, steps=max(args.steps, 1), batches=(args.batch,))
        elif args.only == "vp":
            res = vocab_parallel_section(dev, 1, 0, peak, steps=max(args.steps, 1), batches=(args.batch,))
        elif args.only == "sampler":
            g = torch.Generator(device=dev).manual_seed(1234)
            weights = [(torch.randn(VOCAB, HIDDEN, device=dev, generator=g) * 0.02).half() for _ in range(4)]
            res = sampler_section(dev, weights, steps=max(args.steps, 1), batches=(1, args.batch))
        elif args.only == "groups":
            g = torch.Generator(device=dev).manual_seed(1234)
            weights = [(torch.randn(VOCAB, HIDDEN, device=dev, generator=g) * 0.02).half() for _ in range(2)]
            res = lane_groups_section(dev, weights, steps=max(args.steps, 1))
        elif args.only == "graphed":
            res = graphed_head_section(dev, steps=max(args.steps, 1))
        else:
            res = mixed_section(dev, peak, steps=max(args.steps, 1))
        print(json.dumps({"only": args.only, "result": res}), flush=True)
        return 0

    from gsp import _native
    from gsp import vocab_parallel as vp

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local_rank)
    dev = torch.device("cuda", local_rank)
    xch = None
    if world > 1:
        import torch.distributed as dist
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
        xch = vp.PeerExchange(max_batch=1)
    lo, hi = vp.shard_bounds(VOCAB, world, rank)

    # weight shard(s), hidden state and seeded masks (identical on every rank)
    g = torch.Generator(device=dev).manual_seed(1234 + rank)
    copies = args.copies
    weights = [(torch.randn(hi - lo, HIDDEN, device=dev, generator=g) * 0.02).half() for _ in range(copies)]
    weight = weights[0]
    hidden = torch.randn(1, HIDDEN, device=dev, generator=torch.Generator(device=dev).manual_seed(99)).half()
    masks_np = make_masks(args.masks, args.density, args.pattern, seed=100)
    counts = legal_counts(masks_np)
    masks = torch.from_numpy(masks_np).to(dev)
    local_masks = masks[:, lo // 32:(hi + 31) // 32]
    local_counts = legal_counts_local(masks_np, lo, hi)

    logits = torch.empty(1, hi - lo, device=dev, dtype=torch.float16)
    top_value = torch.empty(1, device=dev, dtype=torch.float32)
    top_index = torch.empty(1, device=dev, dtype=torch.int64)
    top_key = torch.empty(1, device=dev, dtype=torch.int64)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def step(i, mask_rows=local_masks):
        m = mask_rows[i % mask_rows.shape[0]][None]
        w = weights[i % len(weights)]
        if world == 1:
            _native.row_sparse(hidden, w, m, logits=logits, top_value=top_value, top_index=top_index)
        else:
            _native.vocab_parallel("row-sparse", hidden, w, m, xch.peers, rank, xch.max_batch, VOCAB, logits=logits,
                                   top_value=top_value, top_index=top_index, vocab_offset=lo)

    def barrier():
        if world > 1:
            torch.distributed.barrier()
        torch.cuda.synchronize()

    def timed(n, fn, offset, flush_l2=True):
        """Eager steps, each with its own events (µs); with flush_l2, each after
        an L2-flushing write (outside the events)."""
        ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
        for i in range(n):
            if flush_l2:
                flush.zero_()
            ev0[i].record()
            fn(offset + i)
            ev1[i].record()
        torch.cuda.synchronize()
        return [a.elapsed_time(b) * 1e3 for a, b in zip(ev0, ev1)]

    def graph_replays_us(n, fn, min_replays=50, min_seconds=1.0, max_replays=20000):
        """n steps captured in one CUDA graph, replayed at least min_replays
        times and for at least min_seconds of device time; CUDA events around
        every replay (µs per replay, one entry per replay)."""
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for i in range(3):
                fn(i)  # creates this stream's workspace before capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for i in range(n):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        out = []
        while len(out) < max_replays and (len(out) < min_replays or sum(out) < min_seconds * 1e6):
            ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(50)]
            for a, b in ev:
                a.record()
                graph.replay()
                b.record()
            ev[-1][1].synchronize()
            out += [a.elapsed_time(b) * 1e3 for a, b in ev]
        del graph
        return out

    def graph_total_us(n, fn):
        """n steps captured in one CUDA graph; events around one replay (µs)."""
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            for i in range(3):
                fn(i)  # creates this stream's workspace before capture
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            for i in range(n):
                fn(i)
        graph.replay()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        graph.replay()
        b.record()
        b.synchronize()
        del graph
        return a.elapsed_time(b) * 1e3

    # warm-up (untimed)
    for i in range(max(args.warmup, 3)):
        step(i)
    barrier()
    clocks = ClockSampler(local_rank)
    with clocks:
        t_wall = time.perf_counter()
        replay_us = graph_replays_us(args.steps, step)
        barrier()
        t_wall = time.perf_counter() - t_wall
    total_us = max_over_ranks(statistics.median(replay_us), world)
    replays = {"count": len(replay_us), "median_us": statistics.median(replay_us), "min_us": min(replay_us),
               "p90_us": sorted(replay_us)[int(0.9 * (len(replay_us) - 1))],
               "what": (f"the {args.steps} timed steps captured in one CUDA graph and replayed {len(replay_us)} "
                        f"times (>= 50 replays and >= 1 s), CUDA events around each replay; value uses the median "
                        f"replay (max over ranks)")}
    # the last timed step again, eagerly on the same inputs, checked against
    # exact float64 products
    last = args.steps - 1
    step(last)
    parity = exact_check(hidden, weights[last % len(weights)], local_masks[last % local_masks.shape[0]][None], logits,
                         top_index) if world == 1 else None
    steps_idx = [i % args.masks for i in range(args.steps)]
    legal_bytes = float(sum(int(counts[j]) for j in steps_idx)) * HIDDEN * 2
    value = legal_bytes / (total_us * 1e-6) / 1e9
    us_per_step = total_us / args.steps
    cold = None
    if world == 1:
        cold_steps = timed(min(args.steps, 200), step, 0)
        cold = {"us_per_step": statistics.mean(cold_steps), "us_p50": statistics.median(cold_steps),
                "what": "eager steps, 256 MiB L2-flushing write before each, events around each step"}

    # e2e through the C ABI with host buffers: each step's mask and hidden state
    # sit in one pinned staging row, moved to the device by gsp_copy_bytes (an
    # SM-driven copy: a copy-engine transfer's fixed latency dominates at
    # 35 KB); the kernel stores the 16-byte top-1 record straight into pinned
    # host memory (at N > 1 the global record, after the in-kernel exchange).
    local_words = (hi + 31) // 32 - lo // 32
    mask_bytes = local_words * 4
    mask_pad = (mask_bytes + 15) // 16 * 16
    in_bytes = mask_pad + HIDDEN * 2
    host_in = torch.zeros(args.masks, in_bytes, dtype=torch.uint8).pin_memory()
    hidden_bytes = hidden.cpu().view(torch.uint8).reshape(-1)
    for j in range(args.masks):
        host_in[j, :mask_bytes] = torch.from_numpy(
            np.ascontiguousarray(masks_np[j, lo // 32:(hi + 31) // 32])).view(torch.uint8)
        host_in[j, mask_pad:] = hidden_bytes
    dev_in = torch.empty(in_bytes, dtype=torch.uint8, device=dev)
    dev_mask = dev_in[:mask_bytes].view(torch.int32).view(1, local_words)
    dev_hidden = dev_in[mask_pad:].view(torch.float16).view(1, HIDDEN)
    dev_out = torch.empty(2, dtype=torch.int64, device=dev)  # [index, value bits]
    out_index = dev_out[0:1]
    out_value = dev_out[1:2].view(torch.float32)[:1]
    host_top = torch.empty(2, dtype=torch.int64).pin_memory()

    host_index = host_top[0:1]
    host_value = host_top[1:2].view(torch.float32)[:1]

    # one prepared C-ABI call per weight copy (arguments converted once)
    if world == 1:
        calls = [_native.PreparedProjection("gsp_row_sparse_logits", dev_hidden, w, dev_mask, logits=logits,
                                            top_value=host_value, top_index=host_index) for w in weights]
    else:
        calls = [_native.PreparedVocabParallel("row-sparse", dev_hidden, w, dev_mask, xch.peers, rank, xch.max_batch,
                                               VOCAB, logits=logits, top_value=host_value, top_index=host_index,
                                               vocab_offset=lo) for w in weights]

    host_rows = [host_in[j] for j in range(args.masks)]
    if world == 1:
        # one C-ABI call per step: the step recorded once per weight copy as a
        # CUDA graph inside the library (the pinned row's copy, then the
        # projection), replayed with its copy pointed at the step's row
        fused = [_native.PreparedStep(host_rows[0], dev_in, dev_hidden, w, dev_mask, logits=logits,
                                      top_value=host_value, top_index=host_index) for w in weights]
        graphs = [_native.GraphStep(host_rows[0], dev_in, dev_hidden, w, dev_mask, logits=logits,
                                    top_value=host_value, top_index=host_index) for w in weights]

        def e2e_step(i):
            graphs[i % len(graphs)](host_rows[i % args.masks])

        def fused_step(i):
            fused[i % len(fused)](host_rows[i % args.masks])
    else:
        def e2e_step(i):
            _native.copy_bytes(dev_in, host_rows[i % args.masks])
            calls[i % len(calls)]()

    for i in range(3):
        e2e_step(i)
    barrier()
    # one step at a time, as a decode loop runs it: events around the step and
    # a host wait for its result record before the next step is issued
    e2e_steps = []
    for i in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        e2e_step(i)
        b.record()
        b.synchronize()
        int(host_top[0])  # the step's result, read on the host
        e2e_steps.append(a.elapsed_time(b) * 1e3)
    barrier()
    e2e_parts = e2e_breakdown(dev, e2e_step, lambda i: _native.copy_bytes(dev_in, host_rows[i % args.masks]),
                              lambda i: calls[i % len(calls)](), args.steps) if world == 1 else None
    if e2e_parts is not None:  # the same step as two C-ABI calls (copy, then projection)
        def two_calls(i):
            _native.copy_bytes(dev_in, host_rows[i % args.masks])
            calls[i % len(calls)]()
        e2e_parts["two_calls_step_us"] = e2e_breakdown(dev, two_calls, lambda i: None, lambda i: None,
                                                       args.steps)["step_us"]
        e2e_parts["one_call_no_graph_step_us"] = e2e_breakdown(dev, fused_step, lambda i: None, lambda i: None,
                                                               args.steps)["step_us"]
    # the last step's record on the host equals a call on its inputs with device outputs
    last = (args.steps - 1) % len(weights)
    if world == 1:
        _native.row_sparse(dev_hidden, weights[last], dev_mask, top_index=out_index)
    else:
        _native.vocab_parallel("row-sparse", dev_hidden, weights[last], dev_mask, xch.peers, rank, xch.max_batch,
                               VOCAB, top_value=out_value, top_index=out_index, vocab_offset=lo)
    if int(out_index.item()) != int(host_top[0]) or int(host_top[0]) < 0:
        raise RuntimeError("end-to-end step's host record disagrees with the device-output call "
                           "(or the cross-rank exchange timed out)")
    e2e_total = max_over_ranks(sum(e2e_steps), world)
    e2e_value = legal_bytes / (e2e_total * 1e-6) / 1e9
    e2e_graph_us = e2e_graph_replay(dev, weights, host_in, dev_in, dev_hidden, dev_mask, logits, host_value,
                                    host_index, args) if world == 1 else None
    h2d = int(in_bytes)
    d2h = int(dev_out.numel() * 8)

    # roofline of the row-sparse kernel (rank 0's shard at N > 1)
    local_bytes = float(sum(int(local_counts[j]) for j in steps_idx)) * HIDDEN * 2
    kernel_us = us_per_step if world == 1 else None
    peak, peak_src = read_peaks()
    algo_per_launch = local_bytes / args.steps
    if world == 1:
        achieved = algo_per_launch / (kernel_us * 1e-6) / 1e9
        traffic, traffic_src = read_traffic_csv()
        roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                    "frac": achieved / peak, "traffic": traffic, "traffic_source": traffic_src,
                    "kernel": "row_sparse_staged_kernel", "algorithmic_bytes_per_launch": algo_per_launch,
                    "peak_source": peak_src, "avg_launch_us": kernel_us,
                    "all_bytes_per_launch": algo_per_launch + (VOCAB // 32) * 4 + HIDDEN * 2 + VOCAB * 2}
    else:
        roofline = None

    sweep = None
    batched = None
    mixed = None
    sampler_res = None
    graphed = None
    groups = None
    same_gpu_dense = None
    ref_triton = None
    cpu_base = None
    if world == 1 and not args.no_sweep:
        sweep = []
        for pattern in ("uniform", "clustered"):
            for d in DENSITIES:
                mk_np = make_masks(16, d, pattern, seed=200)
                mk = torch.from_numpy(mk_np).to(dev)
                cnt = legal_counts(mk_np)
                n = args.sweep_steps
                t_us = graph_total_us(n, lambda i: step(i, mk))
                ts = timed(min(n, 50), lambda i: step(i, mk), 0)
                lb = float(sum(int(cnt[i % 16]) for i in range(n))) * HIDDEN * 2
                sweep.append({"density": d, "pattern": pattern, "us_per_step": t_us / n,
                              "legal_gbs": lb / (t_us * 1e-6) / 1e9,
                              "frac_of_hbm": lb / (t_us * 1e-6) / 1e9 / peak,
                              "cold_us_per_step": statistics.mean(ts)})
        same_gpu_dense = time_dense_baseline(dev, weight, hidden, masks, args)
        batched = batched_section(dev, weights[:8], peak)
        mixed = mixed_section(dev, peak)
        sampler_res = sampler_section(dev, weights[:8])
        graphed = graphed_head_section(dev)
        groups = lane_groups_section(dev, weights[:8])
        ref_triton = reference_triton_section(dev, args, weights, hidden, masks, us_per_step, batched)
    vp_head = None if args.no_vp else vocab_parallel_section(dev, world, rank, peak)
    if world == 1 and rank == 0 and not args.no_cpu_baseline:
        w_cpu = weight.cpu().numpy()
        h_cpu = hidden.cpu().numpy()
        cpu_base = cpu_baselines(w_cpu, h_cpu, masks_np, args.cpu_seconds, args.density, args.pattern)

    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": us_per_step / 1e3, "us_per_step": us_per_step,
            "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f16", "data": "synthetic",
            "config": workload_config(args),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "us_per_step": e2e_total / args.steps,
                    "graph_replay_us_per_step": e2e_graph_us,
                    "breakdown": e2e_parts,
                    "what": ("eager steps one at a time, events around each and a host wait for the step's result "
                             "before the next: one C-ABI call (gsp_step_graph_launch: the step recorded once per "
                             "weight copy as a CUDA graph inside the library) copies the step's mask and hidden "
                             "state from its pinned staging row to the device (SM-driven copy) and runs the "
                             "projection on weight copy i % copies, storing the 16-byte top-1 record into pinned "
                             "host memory, read by the host (at N > 1: gsp_copy_bytes, then the vocabulary-parallel "
                             "call with the in-kernel cross-rank exchange); "
                             "graph_replay_us_per_step: the same step recorded once per weight copy as a CUDA "
                             "graph and replayed (one GPU)")},
            "gpu_launches": args.steps,
            "timing": replays,
            "parity": parity,
            "roofline": roofline,
            "cpu_baseline": cpu_base,
            "clocks": clocks.summary(),
            "cold": cold,
            "timed_region_wall_s": t_wall,
            "sweep": sweep,
            "batched": batched,
            "mixed": mixed,
            "same_gpu_dense_mask": same_gpu_dense,
            "reference_triton_same_gpu": ref_triton,
            "vocab_parallel_head": vp_head,
            "sampler": sampler_res,
            "graphed_head": graphed,
            "lane_groups": groups,
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        xch.close()
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()
    return 0


def e2e_graph_replay(dev, weights, host_in, dev_in, dev_hidden, dev_mask, logits, host_value, host_index, args):
    """The end-to-end step as a CUDA graph per weight copy (the SM copy of a
    pinned staging row and the C-ABI call storing the top-1 record into pinned
    host memory, recorded once), replayed per step after the step's input is
    written into that graph's staging row; mean µs per step from events around
    each replay."""
    from gsp import _native
    stages = [torch.zeros(host_in.shape[1], dtype=torch.uint8).pin_memory() for _ in weights]
    done = [torch.cuda.Event() for _ in weights]
    cap = torch.cuda.Stream(device=dev)
    cap.wait_stream(torch.cuda.current_stream(dev))
    with torch.cuda.stream(cap):
        calls = [_native.PreparedProjection("gsp_row_sparse_logits", dev_hidden, w, dev_mask, logits=logits,
                                            top_value=host_value, top_index=host_index) for w in weights]
        for j, call in enumerate(calls):
            _native.copy_bytes(dev_in, stages[j])
            call()
    cap.synchronize()
    graphs = []
    for j, call in enumerate(calls):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            _native.copy_bytes(dev_in, stages[j])
            call()
        graphs.append(g)
    n = args.steps
    ev0 = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    ev1 = [torch.cuda.Event(enable_timing=True) for _ in range(n)]
    for i in range(-3, n):
        j = i % len(graphs)
        done[j].synchronize()  # the staging row's previous copy has run
        stages[j].copy_(host_in[i % args.masks])
        if i >= 0:
            ev0[i].record()
        graphs[j].replay()
        if i >= 0:
            ev1[i].record()
        done[j].record()
    torch.cuda.synchronize()
    us = sum(a.elapsed_time(b) * 1e3 for a, b in zip(ev0, ev1)) / n
    del graphs
    return us


def e2e_breakdown(dev, full_step, copy_step, call_step, n: int):
    """Splits the end-to-end step (one GPU): device time of the input copy
    kernel alone, of the prepared projection call alone and of the whole step,
    each with CUDA events and a host wait after every step (medians); the
    host-side issue cost of a step (Python + ctypes + launches, the calls
    queued without waiting); and the wall-clock time of a step including the
    host's wake-up after the result is ready."""
    def events_us(fn):
        ts = []
        for i in range(n):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn(i)
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        return statistics.median(ts)

    def issue_us(fn):
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(n):
            fn(i)
        el = time.perf_counter() - t0
        torch.cuda.synchronize()
        return el / n * 1e6

    def wall_us(fn):
        ts = []
        for i in range(n):
            t0 = time.perf_counter()
            fn(i)
            torch.cuda.current_stream().synchronize()
            ts.append((time.perf_counter() - t0) * 1e6)
        return statistics.median(ts)

    return {"copy_kernel_us": events_us(copy_step), "projection_call_us": events_us(call_step),
            "step_us": events_us(full_step), "host_issue_us_per_step": issue_us(full_step),
            "wall_us_per_step": wall_us(full_step),
            "what": ("medians over the timed steps; *_us: CUDA events around each piece with a host wait after "
                     "each; host_issue: host time to queue one step without waiting; wall: perf_counter around "
                     "a step and the wait for its result")}


def legal_counts_local(masks_np: np.ndarray, lo: int, hi: int) -> np.ndarray:
    from gsp import workloads as wl
    return wl.unpack_bitmask(masks_np, VOCAB)[:, lo:hi].sum(axis=1)


def max_over_ranks(x: float, world: int) -> float:
    if world == 1:
        return x
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
    return float(t.item())


def graph_time_us(dev, n, fn, replays: int = 10):
    """n calls of fn(i) captured in one CUDA graph; events around each of
    `replays` replays; the median replay (us)."""
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(3):
            fn(i)  # creates this stream's workspace before capture
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for i in range(n):
            fn(i)
    graph.replay()
    torch.cuda.synchronize()
    ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(replays)]
    for a, b in ev:
        a.record()
        graph.replay()
        b.record()
    ev[-1][1].synchronize()
    del graph
    return statistics.median(a.elapsed_time(b) * 1e3 for a, b in ev)


def eager_time_us(n, fn):
    """Median of n eager calls, each bracketed by its own events (us)."""
    ts = []
    for i in range(n):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        fn(i)
        b.record()
        b.synchronize()
        ts.append(a.elapsed_time(b) * 1e3)
    return statistics.median(ts)


def batched_section(dev, weights, peak, steps=20, batches=(2, 4, 8, 16, 32)):
    """Batched decode at V=248,320, H=2,048 fp16: every request 0.5% legal in
    <= 16 clustered runs. Times each route, reports the active-tile fraction,
    the block kernel's roofline and whether the B200 cost model picked the
    measured best route."""
    from gsp import _native, triton_runtime as tr
    from gsp import workloads as wl
    import torch.nn.functional as F
    out = []
    ntiles = (VOCAB + 127) // 128
    for batch in batches:
        rng = np.random.default_rng(300 + batch)
        masks_np = [wl.make_batch_mask(rng, batch, VOCAB, [1242] * batch, clustered=True, max_runs=16) for _ in range(8)]
        masks = [torch.from_numpy(m).to(dev) for m in masks_np]
        active = [wl.active_tiles(m, VOCAB) for m in masks_np]
        legal = [wl.unpack_bitmask(m, VOCAB).sum(axis=1) for m in masks_np]
        hidden = torch.randn(batch, HIDDEN, device=dev, generator=torch.Generator(device=dev).manual_seed(batch)).half()
        logits = torch.empty(batch, VOCAB, device=dev, dtype=torch.float16)
        tv = torch.empty(batch, device=dev, dtype=torch.float32)
        ti = torch.empty(batch, device=dev, dtype=torch.int64)
        routes = {"block-sparse": _native.block_gemm, "dense-mask": _native.dense_masked, "row-sparse": _native.row_sparse}
        times = {}
        for name, fn in routes.items():
            times[name] = graph_time_us(dev, steps, lambda i, fn=fn: fn(hidden, weights[i % len(weights)], masks[i % 8],
                                                                         logits=logits, top_value=tv, top_index=ti)) / steps
        try:
            import xgrammar as xgr

            def ref_dense(i):
                lg = F.linear(hidden, weights[i % len(weights)])
                xgr.apply_token_bitmask_inplace(lg, masks[i % 8], vocab_size=VOCAB, backend="triton")
            ref_dense(0)
            times["cublas+xgrammar"] = eager_time_us(10, ref_dense)
        except Exception as exc:  # pragma: no cover - optional comparison
            times["cublas+xgrammar"] = None
        parity = {}
        for name, fn in routes.items():  # one timed step per route, checked
            fn(hidden, weights[0], masks[0], logits=logits, top_value=tv, top_index=ti)
            parity[name] = exact_check(hidden, weights[0], masks[0], logits, ti)
        mean_active = float(np.mean(active))
        block_bytes = mean_active * 128 * HIDDEN * 2
        row_bytes = float(np.mean([l.sum() for l in legal])) * HIDDEN * 2  # legal rows, every request
        best = min(("block-sparse", "dense-mask", "row-sparse"), key=lambda r: times[r])
        choice = tr.choose_route(batch, VOCAB, HIDDEN, 2, legal[0].tolist(), active[0])
        out.append({
            "batch": batch, "active_tile_fraction": mean_active / ntiles,
            "us_per_step": {k: v for k, v in times.items()},
            "block_roofline": {"achieved_gbs": block_bytes / (times["block-sparse"] * 1e-6) / 1e9,
                               "frac": block_bytes / (times["block-sparse"] * 1e-6) / 1e9 / peak,
                               "algorithmic_bytes": block_bytes},
            "row_sparse_roofline": {"achieved_gbs": row_bytes / (times["row-sparse"] * 1e-6) / 1e9,
                                    "frac": row_bytes / (times["row-sparse"] * 1e-6) / 1e9 / peak,
                                    "algorithmic_bytes": row_bytes},
            "dense_roofline_frac": VOCAB * HIDDEN * 2 / (times["dense-mask"] * 1e-6) / 1e9 / peak,
            "speedup_block_vs_cublas_xgrammar": (times["cublas+xgrammar"] / times["block-sparse"]
                                                 if times["cublas+xgrammar"] else None),
            "tokens_per_s": batch / (times[best] * 1e-6),
            "best_route": best, "b200_policy_route": choice, "parity": parity,
        })
    return out


def sampler_section(dev, weights, steps=50, batches=(1, 32)):
    """Fused grammar-conditioned sampler against the unfused pipeline at the
    headline shape (V=248,320, H=2,048 fp16; batch 1: 1% uniform legal tokens,
    batch 32: 0.5% in <= 16 runs per request), graph-timed over the weight
    copies: `fused` = gsp_row_sparse_sample, no logits written; `greedy` = the
    row-sparse kernel with full logits and fused top-1 (the headline step);
    `unfused` = the same kernel writing full logits, then Gumbel-max sampling
    over them in torch (rand, two logs, scale, add, argmax)."""
    from gsp import _native, workloads as wl
    out = []
    temperature = 0.8
    for batch in batches:
        rng = np.random.default_rng(700 + batch)
        if batch == 1:
            masks_np = [wl.make_batch_mask(rng, 1, VOCAB, [VOCAB // 100]) for _ in range(8)]
        else:
            masks_np = [wl.make_batch_mask(rng, batch, VOCAB, [1242] * batch, clustered=True, max_runs=16)
                        for _ in range(8)]
        masks = [torch.from_numpy(m).to(dev) for m in masks_np]
        hidden = torch.randn(batch, HIDDEN, device=dev, generator=torch.Generator(device=dev).manual_seed(5)).half()
        seeds = torch.arange(batch, dtype=torch.int64, device=dev) * 7919 + 17
        logits = torch.empty(batch, VOCAB, device=dev, dtype=torch.float16)
        tv = torch.empty(batch, device=dev, dtype=torch.float32)
        ti = torch.empty(batch, device=dev, dtype=torch.int64)
        tok = torch.empty(batch, device=dev, dtype=torch.int64)
        lse = torch.empty(batch, device=dev, dtype=torch.float32)

        def fused(i):
            _native.row_sparse_sample(hidden, weights[i % len(weights)], masks[i % 8], seeds, i, temperature, tok,
                                      sample_logsumexp=lse, top_value=tv, top_index=ti)

        def greedy(i):
            _native.row_sparse(hidden, weights[i % len(weights)], masks[i % 8], logits=logits, top_value=tv,
                               top_index=ti)

        def unfused(i):
            greedy(i)
            u = torch.rand(batch, VOCAB, device=dev)
            tok.copy_((logits.float() / temperature - torch.log(-torch.log(u))).argmax(-1))

        def fused_block(i):  # the sampler in the tensor-core epilogue, active tiles only
            _native.row_sparse_sample(hidden, weights[i % len(weights)], masks[i % 8], seeds, i, temperature, tok,
                                      sample_logsumexp=lse, top_value=tv, top_index=ti, route="block-sparse")

        fns = [("fused", fused), ("greedy", greedy), ("unfused", unfused)]
        if batch > 1:
            fns.append(("fused_block_sparse", fused_block))
        times = {name: graph_time_us(dev, steps, fn) / steps for name, fn in fns}
        out.append({"batch": batch, "us_per_step": times,
                    "speedup_fused_vs_unfused": times["unfused"] / times["fused"]})
    return out


VP_VOCAB, VP_HIDDEN = 262144, 8192


def vocab_parallel_section(dev, world, rank, peak, steps=10, batches=(1, 32, 128)):
    """Vocabulary-parallel head: V=262,144, H=8,192 bf16, W ~ N(0, 0.01)
    row-sharded over the ranks (this rank's contiguous shard on its GPU),
    batch 1 / 32 / 128, each request 1% legal in <= 16 clustered runs, greedy
    top-1 merged across the ranks inside the kernel (one rank: the plain
    kernels). Every route graph-timed on every rank, max over ranks; the
    per-rank roofline uses each route's algorithmic bytes on the shard."""
    from gsp import _native, triton_runtime as tr, vocab_parallel as vp
    from gsp import workloads as wl
    lo, hi = vp.shard_bounds(VP_VOCAB, world, rank)
    vloc = hi - lo
    g = torch.Generator(device=dev).manual_seed(4321 + rank)
    w = (torch.randn(vloc, VP_HIDDEN, device=dev, generator=g) * 0.01).bfloat16()
    xch = vp.PeerExchange(max_batch=max(batches)) if world > 1 else None
    plain = {"row-sparse": _native.row_sparse, "block-sparse": _native.block_gemm,
             "dense-mask": _native.dense_masked}
    row_bytes = VP_HIDDEN * 2
    out = []
    for batch in batches:
        rng = np.random.default_rng(500 + batch)  # the same masks on every rank
        full = [wl.make_batch_mask(rng, batch, VP_VOCAB, [VP_VOCAB // 100] * batch, clustered=True, max_runs=16)
                for _ in range(4)]
        local_np = [np.ascontiguousarray(m[:, lo // 32:(hi + 31) // 32]) for m in full]
        masks = [torch.from_numpy(m).to(dev) for m in local_np]
        legal = [wl.unpack_bitmask(m, VP_VOCAB)[:, lo:hi].sum(axis=1) for m in full]
        active = [wl.active_tiles(m, vloc) for m in local_np]
        h = torch.randn(batch, VP_HIDDEN, device=dev,
                        generator=torch.Generator(device=dev).manual_seed(600 + batch)).bfloat16()
        tv = torch.empty(batch, device=dev, dtype=torch.float32)
        ti = torch.empty(batch, device=dev, dtype=torch.int64)
        times, fracs = {}, {}
        route_bytes = {"row-sparse": float(np.mean([l.sum() for l in legal])) * row_bytes,
                       "block-sparse": float(np.mean(active)) * 128 * row_bytes,
                       "dense-mask": float(vloc) * row_bytes}
        for route in ("row-sparse", "block-sparse", "dense-mask"):
            def fn(i, route=route):
                m = masks[i % 4]
                if xch is None:
                    plain[route](h, w, m, top_value=tv, top_index=ti)
                else:
                    _native.vocab_parallel(route, h, w, m, xch.peers, rank, xch.max_batch, VP_VOCAB,
                                           top_value=tv, top_index=ti, vocab_offset=lo)
            t = max_over_ranks(synced_graph_time_us(dev, steps, fn, world), world) / steps
            times[route] = t
            fracs[route] = route_bytes[route] / (t * 1e-6) / 1e9 / peak
        parity = None
        if xch is None:  # one GPU: every route once with logits, checked
            parity = {}
            lg = torch.empty(batch, vloc, device=dev, dtype=torch.bfloat16)
            for route, fn in plain.items():
                fn(h, w, masks[0], logits=lg, top_value=tv, top_index=ti)
                parity[route] = exact_check(h, w, masks[0], lg, ti)
            del lg
        best = min(times, key=times.get)
        choice = tr.choose_route(batch, vloc, VP_HIDDEN, 2, legal[0].tolist(), active[0])
        out.append({"batch": batch, "us_per_step": times, "hbm_roofline_frac_per_rank": fracs, "parity": parity,
                    "active_tile_fraction_per_rank": float(np.mean(active)) / ((vloc + 127) // 128),
                    "best_route": best, "b200_policy_route": choice,
                    "tokens_per_s": batch / (times[best] * 1e-6)})
    if xch is not None:
        xch.close()
    return {"vocab": VP_VOCAB, "hidden": VP_HIDDEN, "dtype": "bf16", "ranks": world,
            "outputs": "greedy top-1 (global ids), no logits", "results": out}


def synced_graph_time_us(dev, n, fn, world):
    """Like graph_time_us, with the ranks aligned by a barrier before each
    replay (their kernels wait on one another inside the exchange)."""
    s = torch.cuda.Stream(device=dev)
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for i in range(2):
            fn(i)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        for i in range(n):
            fn(i)
    if world > 1:
        torch.distributed.barrier()
    graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    graph.replay()
    b.record()
    b.synchronize()
    del graph
    return a.elapsed_time(b) * 1e3


def mixed_section(dev, peak, steps=10):
    """Mixed-density dispatcher sweep: V=151,936, H=1,024 bf16, batch 64;
    a seeded mix of near-unconstrained (95% uniform) and constrained (0.2% in
    <= 16 runs) requests. Reports each route's time and both policies' picks."""
    from gsp import _native, triton_runtime as tr
    from gsp import workloads as wl
    vocab, hidden, batch = 151936, 1024, 64
    g = torch.Generator(device=dev).manual_seed(5)
    weights = [(torch.randn(vocab, hidden, device=dev, generator=g) * 0.02).bfloat16() for _ in range(4)]
    h = torch.randn(batch, hidden, device=dev, generator=g).bfloat16()
    logits = torch.empty(batch, vocab, device=dev, dtype=torch.bfloat16)
    tv = torch.empty(batch, device=dev, dtype=torch.float32)
    ti = torch.empty(batch, device=dev, dtype=torch.int64)
    out = []
    for frac in (0.0, 0.25, 0.5, 0.75, 1.0):
        rng = np.random.default_rng(int(frac * 100))
        masks_np = [wl.mixed_batch_mask(rng, batch, vocab, frac) for _ in range(4)]
        masks = [torch.from_numpy(m).to(dev) for m in masks_np]
        times = {}
        for name, fn in (("block-sparse", _native.block_gemm), ("dense-mask", _native.dense_masked),
                         ("row-sparse", _native.row_sparse)):
            times[name] = graph_time_us(dev, steps, lambda i, fn=fn: fn(h, weights[i % 4], masks[i % 4], logits=logits,
                                                                       top_value=tv, top_index=ti)) / steps
        parity = {}
        for name, fn in (("block-sparse", _native.block_gemm), ("dense-mask", _native.dense_masked),
                         ("row-sparse", _native.row_sparse)):
            fn(h, weights[0], masks[0], logits=logits, top_value=tv, top_index=ti)
            parity[name] = exact_check(h, weights[0], masks[0], logits, ti)
        best = min(times, key=times.get)
        fwf = tr.full_word_fraction_cpu(torch.from_numpy(masks_np[0]))
        ref_route = tr._reference_route(batch, fwf, 0.80)
        stats_legal = wl.unpack_bitmask(masks_np[0], vocab).sum(axis=1).tolist()
        b200_route = tr.choose_route(batch, vocab, hidden, 2, stats_legal, wl.active_tiles(masks_np[0], vocab))
        out.append({"constrained_fraction": frac, "us_per_step": times, "best_route": best,
                    "reference_policy_route": ref_route, "reference_policy_us": times[ref_route],
                    "b200_policy_route": b200_route, "b200_policy_us": times[b200_route],
                    "tokens_per_s_best": batch / (times[best] * 1e-6), "parity": parity})
    del weights
    return out


def graphed_head_section(dev, steps=20):
    """Device-side mask path at the mixed shape (V=151,936, H=1,024 bf16,
    batch 64), one mask per constrained fraction. GraphedGrammarHead: the head
    as one CUDA graph (device route selector, SWITCH node, chosen projection
    with fused top-1), timed with CUDA events over `steps` back-to-back
    replays; the pinned-mask host-to-device copy (1.2 MB) timed alone on the
    copy stream (in a decode loop it overlaps the transformer layers), and
    staged copy + replay back to back (nothing to overlap with here). Against
    the host-decided dispatch (policy "b200": device statistics read back,
    route chosen on the host) and the eager device selector (policy "device":
    4-byte route read back), wall clock over `steps` calls."""
    import time
    from gsp import triton_runtime as tr
    from gsp import workloads as wl
    from gsp.graphed import GraphedGrammarHead
    vocab, hidden, batch = 151936, 1024, 64
    g = torch.Generator(device=dev).manual_seed(7)
    w = (torch.randn(vocab, hidden, device=dev, generator=g) * 0.02).bfloat16()
    h = torch.randn(batch, hidden, device=dev, generator=g).bfloat16()
    head = GraphedGrammarHead(w, batch)
    head.hidden.copy_(h)

    def events_us(fn, stream=None):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s = stream or torch.cuda.current_stream(dev)
        for _ in range(3):
            fn()
        torch.cuda.synchronize()
        e0.record(s)
        for _ in range(steps):
            fn()
        e1.record(s)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) * 1e3 / steps

    out = []
    for frac in (0.0, 0.5, 1.0):
        rng = np.random.default_rng(int(frac * 100) + 11)
        n_con = int(round(frac * batch))
        legal = np.zeros((batch, vocab), dtype=bool)
        for b in range(batch):
            ids = (wl.clustered_legal_ids(rng, vocab, int(0.002 * vocab), 16) if b < n_con
                   else wl.uniform_legal_ids(rng, vocab, int(0.95 * vocab)))
            legal[b, ids] = True
        mask_np = wl.pack_bitmask(legal)
        head.wait_mask_copied()
        head.mask_host.copy_(torch.from_numpy(mask_np))
        head.stage_mask()
        head.step()
        torch.cuda.synchronize()
        route = head.route_names()[0]
        graph_us = events_us(head.step)

        def copy_only():
            head.mask.copy_(head.mask_host, non_blocking=True)
        with torch.cuda.stream(head.copy_stream):
            copy_us = events_us(copy_only, head.copy_stream)

        def staged():
            head.stage_mask()
            head.step()
        staged_us = events_us(staged)
        mask_dev = torch.from_numpy(mask_np).to(dev)
        eager = {}
        for policy in ("b200", "device"):
            for _ in range(3):
                tr.adaptive_grammar_logits(h, w, mask_dev, policy=policy)
            torch.cuda.synchronize()
            t0 = time.perf_counter()
            for _ in range(steps):
                _, r = tr.adaptive_grammar_logits(h, w, mask_dev, policy=policy)
            torch.cuda.synchronize()
            eager[policy] = {"us_per_step": (time.perf_counter() - t0) * 1e6 / steps, "route": r}
        fn = {"row-sparse": _native_fn("row_sparse"), "block-sparse": _native_fn("block_gemm"),
              "dense-mask": _native_fn("dense_masked")}[route]
        direct_us = graph_time_us(dev, steps, lambda i: fn(h, w, mask_dev, logits=head.out.logits,
                                                            top_value=head.out.top_value,
                                                            top_index=head.out.top_index)) / steps
        out.append({"constrained_fraction": frac, "route": route, "graphed_head_us": graph_us,
                    "chosen_route_alone_us": direct_us, "mask_h2d_copy_us": copy_us,
                    "staged_copy_then_head_us": staged_us, "mask_bytes": int(mask_np.nbytes),
                    "host_b200_policy": eager["b200"], "eager_device_policy": eager["device"]})
    del head, w
    return out


def lane_groups_section(dev, weights, steps=10):
    """Lane grouping (grouped_grammar_logits) at V=248,320, H=2,048 fp16, batch
    32: `n_clustered` requests with 20% of the vocabulary in one run (the same
    region) batched with scattered requests (0.5% uniform), and the uniform
    batch of the batched section (0.5% in <= 16 runs) where a split does not
    pay. Grouped path (plan, read-back, gathers, two routes, un-permute) and
    each single route, wall clock per call with the result synchronised;
    greedy top-1 only (no logits), weight copy i % len(weights)."""
    import time
    from gsp import _native, triton_runtime as tr
    from gsp import workloads as wl
    batch = 32
    out = []
    cases = []
    for n_cl in (4, 8):
        rng = np.random.default_rng(900 + n_cl)
        sc = wl.make_batch_mask(rng, batch - n_cl, VOCAB, [1242] * (batch - n_cl))
        cl = np.repeat(wl.make_batch_mask(rng, 1, VOCAB, [VOCAB // 5], clustered=True, max_runs=1), n_cl, axis=0)
        m = np.concatenate([sc, cl])
        cases.append((f"{batch - n_cl} scattered 0.5% + {n_cl} clustered 20%", m[rng.permutation(batch)]))
    rng = np.random.default_rng(332)
    cases.append(("32 x 0.5% in <= 16 runs", wl.make_batch_mask(rng, batch, VOCAB, [1242] * batch, clustered=True,
                                                                 max_runs=16)))
    h = torch.randn(batch, HIDDEN, device=dev, generator=torch.Generator(device=dev).manual_seed(3)).half()
    tv = torch.empty(batch, device=dev)
    ti = torch.empty(batch, device=dev, dtype=torch.int64)

    def wall_us(fn):
        for i in range(3):
            fn(i)
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(steps):
            fn(i)
            torch.cuda.synchronize()
        return (time.perf_counter() - t0) * 1e6 / steps

    for name, mask_np in cases:
        md = torch.from_numpy(mask_np).to(dev)
        res = tr.grouped_grammar_logits(h, weights[0], md, return_logits=False)
        t = {"grouped": wall_us(lambda i: tr.grouped_grammar_logits(h, weights[i % len(weights)], md,
                                                                    return_logits=False))}
        for route, fn in (("row-sparse", _native.row_sparse), ("block-sparse", _native.block_gemm),
                          ("dense-mask", _native.dense_masked)):
            t[route] = wall_us(lambda i, fn=fn: fn(h, weights[i % len(weights)], md, top_value=tv, top_index=ti))
        best_single = min(("row-sparse", "block-sparse", "dense-mask"), key=lambda r: t[r])
        out.append({"case": name, "plan_routes": list(res.plan["routes"]), "split": res.plan["split"],
                    "modelled_us": {"single": res.plan["single_us"], "split": res.plan["split_us"]},
                    "us_per_call": t, "best_single_route": best_single,
                    "speedup_vs_best_single": t[best_single] / t["grouped"]})
    return out


def _native_fn(name):
    from gsp import _native
    return getattr(_native, name)


def time_dense_baseline(dev, weight, hidden, masks, args):
    """Same-GPU dense LM head + mask as the reference's dense route runs it:
    cuBLAS (F.linear) then xgrammar's Triton mask kernel."""
    try:
        import xgrammar as xgr
        import torch.nn.functional as F
    except Exception as exc:  # pragma: no cover - optional comparison
        return {"unavailable": str(exc)}
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def dense(i):
        lg = F.linear(hidden, weight)
        xgr.apply_token_bitmask_inplace(lg, masks[i % masks.shape[0]][None], vocab_size=VOCAB, backend="triton")
        return lg

    try:
        for i in range(3):
            dense(i)
        torch.cuda.synchronize()
        ts = []
        for i in range(50):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            dense(i)
            b.record()
            b.synchronize()
            ts.append(a.elapsed_time(b) * 1e3)
        return {"us_per_step": statistics.median(ts), "what": "F.linear (cuBLAS) + xgrammar triton mask, batch 1"}
    except Exception as exc:  # pragma: no cover
        return {"unavailable": f"{type(exc).__name__}: {exc}"[:200]}


if __name__ == "__main__":
    sys.exit(main())
