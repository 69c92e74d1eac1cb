"""WKV fwd+bwd benchmark on B200 (SpikeGPT RWKV-4 time-mix recurrence).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl native|reference]

One step = one forward and one backward pass of the WKV op over one batch of
synthetic config-1 inputs (B=64, T=1024, C=512, bf16 I/O, k/v ~ 4*N(0,1),
time_decay ~ U(-5,1), time_first ~ U(-1,1), grad_y ~ N(0,1)).

* value: algorithmic bytes per step (16 B/element for bf16: fwd reads k,v and
  writes y; bwd reads k,v,grad_y and writes grad_k,grad_v) times steps, divided
  by the device time of the K timed steps, with inputs resident in HBM, through
  the C ABI (libspikegpt_wkv.so). Inputs are larger than L2 (201 MB of inputs
  per step, ~470 MB touched), so no L2 flush is inserted.
* e2e: the same metric through the public torch ops (myelin::wkv_forward_bf16io
  and myelin::wkv_backward_bf16io) with pinned host buffers: every step copies
  k, v, grad_y, time_decay, time_first host->device and y, grad_k, grad_v and the
  two per-channel grads device->host inside the timed region.
* roofline: the kernel with the largest share of device time, timed per launch
  with CUDA events on its stream during the timed region.
* cpu_baseline: the CPU oracle port (oracle/wkv_oracle.c, float32, all host
  threads) on a bounded sample of the same workload, rank 0 at N=1.

Multi-GPU (torchrun): the batch shards across ranks with no data-path
collective (every (b, c) lane is independent): each rank runs the config-1
batch on its own GPU (weak scaling); timing is the max over ranks.

--impl reference times the reference's CPU implementation of the path (the
oracle port, since the reference is Python and cannot travel) on the same
config, rank 0 only.
"""

from __future__ import annotations

import argparse
import json
import os
import re
import statistics
import subprocess
import sys
import threading
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "spikegpt-myelin_b200"))
sys.path.insert(0, str(ROOT))
# The reference itself (baseline/install_ref.py puts it in the git-ignored
# baseline/_ref; its absent dependency myelin is replaced by the test-only
# stand-in). Used only by the reference arm and the incumbent leg.
REF_DIR = ROOT / "baseline" / "_ref"
MYELIN_SHIM = ROOT / "tests" / "golden" / "_myelin_shim"

BYTES_PER_ELEM = {"bf16": 16, "fp16": 16, "fp32": 32}  # fwd 3 tensors + bwd 5 tensors
WORKLOADS = {
    "cfg1": dict(B=64, T=1024, C=512, dtype="bf16", kscale=4.0, desc="config 1: B=64 T=1024 C=512 bf16, k/v x4"),
    "cfg1-fp32": dict(B=64, T=1024, C=512, dtype="fp32", kscale=4.0, desc="config 1 with fp32 I/O"),
    "cfg2": dict(B=24, T=3072, C=512, dtype="bf16", kscale=4.0, desc="config 2: B=24 T=3072 C=512 bf16, k/v x4"),
    "cfg2b-1": dict(B=1, T=3072, C=512, dtype="bf16", kscale=4.0, desc="config 2b: B=1 T=3072 C=512 bf16"),
    "cfg2b-2": dict(B=2, T=3072, C=512, dtype="bf16", kscale=4.0, desc="config 2b: B=2 T=3072 C=512 bf16"),
    "cfg2b-4": dict(B=4, T=3072, C=512, dtype="bf16", kscale=4.0, desc="config 2b: B=4 T=3072 C=512 bf16"),
    "cfg2b-8": dict(B=8, T=3072, C=512, dtype="bf16", kscale=4.0, desc="config 2b: B=8 T=3072 C=512 bf16"),
    "cfg2-b12": dict(B=12, T=3072, C=512, dtype="bf16", kscale=4.0,
                     desc="long context B=12 T=3072 C=512 bf16 (the reference's published row)"),
    "cfg1-b1": dict(B=1, T=1024, C=512, dtype="bf16", kscale=4.0, desc="B=1 T=1024 C=512 bf16"),
    "cfg1-b2": dict(B=2, T=1024, C=512, dtype="bf16", kscale=4.0, desc="B=2 T=1024 C=512 bf16"),
    "cfg1-b4": dict(B=4, T=1024, C=512, dtype="bf16", kscale=4.0, desc="B=4 T=1024 C=512 bf16"),
    "cfg1-b8": dict(B=8, T=1024, C=512, dtype="bf16", kscale=4.0,
                    desc="B=8 T=1024 C=512 bf16 (the per-GPU batch of config 3 on 8 GPUs)"),
    "cfg1-b12": dict(B=12, T=1024, C=512, dtype="bf16", kscale=4.0,
                     desc="B=12 T=1024 C=512 bf16 (the reference's published row)"),
    "cfg1-b24": dict(B=24, T=1024, C=512, dtype="bf16", kscale=4.0,
                     desc="B=24 T=1024 C=512 bf16 (the reference's published row)"),
    # recurrent (generation) step: B decode streams, one token each per step,
    # bf16 keys/values with a float32 state (the autocast case)
    "decode": dict(kind="step", B=16384, T=1, C=512, dtype="bf16", state="fp32", kscale=4.0,
                   desc="recurrent step: B=16384 streams x C=512, bf16 k/v, float32 state"),
}
WORKLOADS["lif"] = dict(kind="lif", B=64, T=1024, C=512, dtype="bf16", kscale=1.5,
                        desc="LIF fwd+bwd: B=64 T=1024 C=512 bf16 (a SpikeGPT-41M block activation)")
WORKLOADS["train"] = dict(kind="train", model="41m", global_batch=64, T=1024, zipf=1.1,
                          desc="config 3: SpikeGPT-41M train step (12L/512d/V=256/ctx1024), global batch 64, "
                               "bf16 autocast, AdamW wd 0.1")
WORKLOADS["train216m"] = dict(kind="train", model="216m", global_batch=32, T=1024, zipf=1.05,
                              desc="config 4: 216M-class SpikeGPT train step (18L/768d/V=50257/ctx1024), "
                                   "global batch 32, bf16 autocast, AdamW wd 0.1")
WORKLOADS["rwkv7"] = dict(kind="rwkv7", B=16, T=1024, H=12, dtype="fp32",
                          desc="config 4 extra: RWKV-7 DPLR forward, H=12 heads of 64, B=16, T=1024, float32")
RWKV7_METRIC = "RWKV-7 DPLR forward algorithmic HBM throughput"
LIF_METRIC = "LIF fwd+bwd algorithmic HBM throughput"
TRAIN_METRIC = "SpikeGPT-41M train tokens/s"
TRAIN_METRICS = {"41m": TRAIN_METRIC, "216m": "SpikeGPT-216M train tokens/s"}
PEAKS_FALLBACK_TFLOPS = 1590.0
STEP_METRIC = "WKV recurrent step algorithmic HBM throughput"
STEP_BYTES = {"bf16": 2, "fp16": 2, "fp32": 4}
METRIC = "WKV fwd+bwd algorithmic HBM throughput"
TRAIN_LEG_STEPS, TRAIN_LEG_WARMUP = 20, 5  # the train_step object of the op bench line
PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "source": "fallback"}


def parse_args():
    ap = argparse.ArgumentParser(description=__doc__, formatter_class=argparse.RawDescriptionHelpFormatter)
    ap.add_argument("--gpus", type=int, default=int(os.environ.get("WORLD_SIZE", "1")))
    ap.add_argument("--steps", type=int, default=3000)
    ap.add_argument("--warmup", type=int, default=20)
    ap.add_argument("--impl", choices=("native", "reference"), default="native")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="cfg1")
    ap.add_argument("--e2e-steps", type=int, default=20)
    ap.add_argument("--e2e-chunks", type=int, default=1, help="batch chunks streamed per e2e step")
    ap.add_argument("--profile", action="store_true", help="device loop only (for ncu): no CPU leg, e2e or clocks")
    ap.add_argument("--no-state", action="store_true",
                    help="time the self-contained op pair (backward re-runs the forward sweep)")
    ap.add_argument("--eager", action="store_true",
                    help="train workloads: launch the step's kernels eagerly instead of replaying a CUDA graph")
    ap.add_argument("--overlap", action="store_true",
                    help="train workloads: all-reduce the gradients in buckets during the backward instead of once "
                         "after it")
    ap.add_argument("--micro-batches", type=int, default=None,
                    help="train workloads: run each rank's batch as this many micro-batches on their own streams "
                         "(default: 2 for 8 to 16 sequences per rank, else 1, as measured on one B200)")
    ap.add_argument("--global-batch", type=int, default=None,
                    help="train workloads: override the global batch (e.g. the per-rank share of an N-GPU run on one GPU)")
    ap.add_argument("--no-train-leg", dest="train_leg", action="store_false",
                    help="WKV workloads: skip the SpikeGPT-41M train-step object of the line")
    ap.add_argument("--no-incumbent", dest="incumbent", action="store_false",
                    help="WKV workloads: skip timing the reference's Triton WKV (incumbent object)")
    ap.add_argument("--incumbent-child", action="store_true", help=argparse.SUPPRESS)
    ap.add_argument("--sweep-segments", default="", metavar="LIST",
                    help="WKV workloads: time the op pair once per forced segment count (e.g. 1,2,4,8) and print "
                         "one JSON line each")
    ap.add_argument("--kernel-split", type=int, default=0, metavar="TOP",
                    help="train workloads: after timing, print the TOP kernels of two eager steps by device time "
                         "(torch profiler, CUDA activity) to stderr")
    return ap.parse_args()


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        d["source"] = "measured"
        return d
    return dict(PEAKS_FALLBACK)


def make_inputs(wl: dict, seed: int):
    """Seeded synthetic inputs with the config's distributions (numpy PCG64)."""
    rng = np.random.default_rng(seed)
    b, t, c = wl["B"], wl["T"], wl["C"]
    k = (rng.standard_normal((b, t, c), dtype=np.float32) * wl["kscale"]).astype(np.float32)
    v = (rng.standard_normal((b, t, c), dtype=np.float32) * wl["kscale"]).astype(np.float32)
    td = rng.uniform(-5.0, 1.0, c).astype(np.float32)
    tf = rng.uniform(-1.0, 1.0, c).astype(np.float32)
    gy = rng.standard_normal((b, t, c), dtype=np.float32)
    return k, v, td, tf, gy


# ------------------------------------------------------------------ clocks


class ClockSampler:
    """nvidia-smi clock/throttle samples for one GPU, with host timestamps."""

    FIELDS = (
        "clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
        "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
        "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap"
    )

    def __init__(self, gpu_index: int, period_ms: int = 100):
        self.samples: list[tuple[float, list[str]]] = []
        self.proc = None
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(gpu_index), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", str(period_ms)],
                stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True,
            )
        except OSError:
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            self.samples.append((time.time(), [x.strip() for x in line.split(",")]))

    def stop(self):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, t0: float, t1: float) -> dict:
        rows = [s for ts, s in self.samples if t0 <= ts <= t1 and len(s) >= 8]
        if not rows:  # very short region: take the samples nearest to it
            rows = [s for ts, s in self.samples if t0 - 0.3 <= ts <= t1 + 0.3 and len(s) >= 8]
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        sm = [num(r[0]) for r in rows if num(r[0]) is not None]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[4:8], strict=False) if v.lower().startswith("active")})
        power = [num(r[2]) for r in rows if num(r[2]) is not None]
        return {
            "sm_mhz": statistics.median(sm) if sm else None,
            "sm_max_mhz": num(rows[0][1]),
            "reasons": reasons,
            "power_w_max": max(power) if power else None,
            "samples": len(rows),
        }


# -------------------------------------------------------------- CPU legs


def cpu_oracle_throughput(wl: dict, *, seconds: float = 10.0, steps: int | None = None, warmup: int = 0):
    """Time the float32 CPU oracle (oracle/wkv_oracle.c) fwd+bwd on one batch
    row of the workload per step with all host threads."""
    from oracle import oracle

    k, v, td, tf, gy = make_inputs(dict(wl, B=1), seed=0)
    threads = os.cpu_count() or 1
    w = -np.exp(td.astype(np.float64)).astype(np.float32)
    run = lambda: (oracle.forward(k, v, td, tf, dtype=np.float32, threads=threads),  # noqa: E731
                   oracle.backward(gy, w, tf, k, v, dtype=np.float32, threads=threads))
    for _ in range(warmup):
        run()
    n = 0
    t0 = time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if (steps is not None and n >= steps) or (steps is None and el >= seconds):
            break
    elems = wl["T"] * wl["C"] * n
    value = BYTES_PER_ELEM[wl["dtype"]] * elems / el / 1e9
    return {
        "value": value,
        "unit": "GB/s",
        "cores": threads,
        "kind": "port",
        "sample": f"{n} x (1 of {wl['B']} batch rows: T={wl['T']} C={wl['C']}), float32, {el:.1f} s",
        "host_cpus": os.cpu_count(),
    }


def reference_available() -> bool:
    return (REF_DIR / "spikegpt" / "language.py").exists()


def _import_reference_language():
    for p in (str(REF_DIR), str(MYELIN_SHIM)):
        if p not in sys.path:
            sys.path.insert(0, p)
    import spikegpt.language as language

    return language


def reference_cpu_throughput(wl: dict, *, steps: int, warmup: int, min_seconds: float = 5.0):
    """Time the reference's own CPU WKV path, ``weighted_key_value`` (the
    associative scan of src/spikegpt/language.py:452-527, what SpikeTimeMix
    runs off CUDA), forward + autograd backward in float32 on all host threads,
    one batch row of the workload per step, for at least ``steps`` steps and
    ``min_seconds``."""
    import torch

    language = _import_reference_language()
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    k, v, td, tf, gy = make_inputs(dict(wl, B=1), seed=0)
    leaves = [torch.tensor(x, requires_grad=True) for x in (k, v, td, tf)]
    gyt = torch.tensor(gy)

    def run():
        for x in leaves:
            x.grad = None
        language.weighted_key_value(*leaves).backward(gyt)

    for _ in range(max(1, warmup)):
        run()
    n = 0
    t0 = time.perf_counter()
    while True:
        run()
        n += 1
        el = time.perf_counter() - t0
        if n >= steps and el >= min_seconds:
            break
    value = BYTES_PER_ELEM[wl["dtype"]] * wl["T"] * wl["C"] * n / el / 1e9
    return {
        "value": value,
        "unit": "GB/s",
        "cores": torch.get_num_threads(),
        "kind": "reference",
        "sample": f"{n} x (1 of {wl['B']} batch rows: T={wl['T']} C={wl['C']}), float32 forward + backward "
                  f"of the reference's weighted_key_value (associative scan, language.py:452-527), {el:.1f} s",
        "host_cpus": os.cpu_count(),
    }


def run_incumbent_child(args, wl):
    """Child process: the reference's own Triton WKV kernels (src/spikegpt/
    wkv_triton.py, wkv_bf16.py) on this GPU, through its public wrappers and
    autograd, as its model calls them. A separate process because the
    reference registers the same myelin:: op names this package does."""
    os.environ["MYELIN_SHIM_HAS_TRITON"] = "1"
    import torch

    for p in (str(REF_DIR), str(MYELIN_SHIM)):
        sys.path.insert(0, p)
    from spikegpt.wkv_bf16 import weighted_key_value_triton_bf16io
    from spikegpt.wkv_triton import weighted_key_value_triton

    dev = torch.device("cuda", 0)
    k_np, v_np, td_np, tf_np, gy_np = make_inputs(wl, seed=0)
    k = torch.as_tensor(k_np).to(dev, torch.bfloat16)
    v = torch.as_tensor(v_np).to(dev, torch.bfloat16)
    gy = torch.as_tensor(gy_np).to(dev, torch.bfloat16)
    td = torch.as_tensor(td_np).to(dev)
    tf = torch.as_tensor(tf_np).to(dev)
    elems = k.numel()
    out = {"workload": wl["desc"], "gpu": torch.cuda.get_device_name(dev)}
    for name, fn in (("bf16io", weighted_key_value_triton_bf16io), ("fp32io_fed_bf16", weighted_key_value_triton)):
        leaves = [x.detach().clone().requires_grad_() for x in (k, v, td, tf)]

        def step(with_backward=True):
            y = fn(*leaves)
            if with_backward:
                y.backward(gy)

        for _ in range(3):
            step()
        torch.cuda.synchronize(dev)
        res = {}
        for label, bwd, steps in (("fwd_bwd", True, args.steps), ("fwd", False, args.steps)):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                if bwd:
                    step(True)
                else:
                    with torch.no_grad():
                        step(False)
            e1.record()
            torch.cuda.synchronize(dev)
            res[f"{label}_ms"] = e0.elapsed_time(e1) / steps
        res["gbs"] = BYTES_PER_ELEM[wl["dtype"]] * elems / (res["fwd_bwd_ms"] * 1e-3) / 1e9
        out[name] = res
    print(json.dumps(out), flush=True)


def incumbent_leg(args, wl) -> dict:
    """The reference's Triton WKV on this GPU (run_incumbent_child in a
    subprocess), or why it could not run."""
    if not reference_available():
        return {"unavailable": "baseline/_ref has no reference install (baseline/install_ref.py)"}
    try:
        import triton  # noqa: F401
    except ImportError:
        return {"unavailable": "triton is not installed"}
    cmd = [sys.executable, str(ROOT / "bench.py"), "--incumbent-child", "--workload", args.workload,
           "--steps", str(max(5, min(args.steps, 50)))]
    try:
        r = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    except subprocess.TimeoutExpired:
        return {"unavailable": "the incumbent child did not finish in 600 s"}
    lines = [ln for ln in r.stdout.splitlines() if ln.startswith("{")]
    if r.returncode != 0 or not lines:
        tail = (r.stderr or r.stdout).strip().splitlines()[-1:] or ["no output"]
        return {"unavailable": f"rc={r.returncode}: {tail[0][:200]}"}
    d = json.loads(lines[-1])
    d["method"] = ("reference wrappers (weighted_key_value_triton_bf16io / weighted_key_value_triton) forward + "
                   "autograd backward on resident bf16 inputs, CUDA events, mean over the steps")
    return d


# ------------------------------------------------------------- native arm


def native_config(wl: dict, b: int, t: int, c: int, world: int) -> dict:
    """The config keys both arms of the WKV workloads report."""
    mb = 3 * BYTES_PER_ELEM[wl["dtype"]] // 8 * b * t * c / 1e6
    return {
        "workload": wl["desc"],
        "B_per_gpu": b,
        "T": t,
        "C": c,
        "global_batch": b * world,
        "parallelism": f"{world} batch-sharded replica(s), no data-path collective",
        "l2": (f"inputs larger than L2 ({mb:.0f} MB of k,v,grad_y read per step); no flush" if mb > 126 else
               f"inputs ({mb:.1f} MB of k,v,grad_y per step) fit in the 126 MB L2; no flush: warm-L2 figure"),
    }


def run_native(args, wl):
    import torch
    import torch.distributed as dist

    import spikegpt_b200
    from spikegpt_b200 import _capi
    from spikegpt_b200.sharding import max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)

    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["dtype"]]
    code = {"bf16": _capi.DTYPE_BF16, "fp16": _capi.DTYPE_F16, "fp32": _capi.DTYPE_F32}[wl["dtype"]]
    b, t, c = wl["B"], wl["T"], wl["C"]
    k_np, v_np, td_np, tf_np, gy_np = make_inputs(wl, seed=rank)
    k = torch.as_tensor(k_np).to(dev, tdt)
    v = torch.as_tensor(v_np).to(dev, tdt)
    gy = torch.as_tensor(gy_np).to(dev, tdt)
    td = torch.as_tensor(td_np).to(dev)
    tf = torch.as_tensor(tf_np).to(dev)
    w = -torch.exp(td)
    y = torch.empty_like(k)
    gk, gv = torch.empty_like(k), torch.empty_like(k)
    gtd, gtf = torch.empty_like(td), torch.empty_like(td)
    lib = _capi.lib()
    fws_n = int(lib.wkv_forward_workspace_size(code, b, t, c))
    bws_n = int(lib.wkv_backward_workspace_size(code, b, t, c))
    st_n = int(lib.wkv_state_size(code, b, t, c))
    fws = torch.empty(max(fws_n, 1), dtype=torch.uint8, device=dev)
    bws = torch.empty(max(bws_n, 1), dtype=torch.uint8, device=dev)
    state = torch.empty(max(st_n, 16), dtype=torch.uint8, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    # The training path: the forward keeps the recurrence state (every 16 steps)
    # and the backward consumes it, as autograd does through the model-facing
    # wrappers. --no-state times the self-contained op pair instead.
    def step_state():
        _capi.check(lib.wkv_forward_with_state(code, k.data_ptr(), v.data_ptr(), td.data_ptr(), tf.data_ptr(),
                                               y.data_ptr(), state.data_ptr(), st_n, b, t, c,
                                               fws.data_ptr(), fws_n, sp), "wkv_forward_with_state")
        _capi.check(lib.wkv_backward_from_state(code, gy.data_ptr(), w.data_ptr(), tf.data_ptr(), k.data_ptr(),
                                                v.data_ptr(), state.data_ptr(), st_n, gk.data_ptr(), gv.data_ptr(),
                                                gtd.data_ptr(), gtf.data_ptr(), b, t, c, bws.data_ptr(), bws_n, sp),
                    "wkv_backward_from_state")

    def step_plain():
        _capi.check(lib.wkv_forward(code, k.data_ptr(), v.data_ptr(), td.data_ptr(), tf.data_ptr(), y.data_ptr(),
                                    b, t, c, fws.data_ptr(), fws_n, sp), "wkv_forward")
        _capi.check(lib.wkv_backward(code, gy.data_ptr(), w.data_ptr(), tf.data_ptr(), k.data_ptr(), v.data_ptr(),
                                     gk.data_ptr(), gv.data_ptr(), gtd.data_ptr(), gtf.data_ptr(),
                                     b, t, c, bws.data_ptr(), bws_n, sp), "wkv_backward")

    step = step_plain if args.no_state else step_state

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    sampler = None if args.profile else ClockSampler(local)
    time.sleep(0.3 if sampler else 0)
    _capi.timing_collect()
    _capi.timing_enable(True)
    launches0 = sum(_capi.launch_counts().values())
    barrier()
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    host1 = time.time()
    barrier()
    _capi.timing_enable(False)
    launches = sum(_capi.launch_counts().values()) - launches0
    per_kernel = _capi.timing_collect()
    ms = ev0.elapsed_time(ev1)
    ms = max_over_ranks(ms, dev)
    if sampler:
        time.sleep(0.25)
        sampler.stop()
    clocks = sampler.summary(host0, host1) if sampler else None

    elems = b * t * c
    step_bytes = BYTES_PER_ELEM[wl["dtype"]] * elems
    value = step_bytes * args.steps * world / (ms * 1e-3) / 1e9

    # roofline of the dominant kernel (largest share of device time)
    io_bytes = BYTES_PER_ELEM[wl["dtype"]] // 8  # bytes of one element of one tensor
    alg_per_launch = {
        "wkv_fwd_kernel<y>": 3 * io_bytes * elems,       # read k, v; write y
        "wkv_bwd_kernel<grad>": 5 * io_bytes * elems,    # read k, v, gy; write gk, gv
        "wkv_fwd_kernel<state>": 0,                      # recompute: no algorithmic bytes
    }
    kernels = {n: {"ms_per_launch": tot / cnt, "launches": cnt, "share": None}
               for n, (tot, cnt) in per_kernel.items() if cnt > 0}
    total_kernel_ms = sum(tot for tot, cnt in per_kernel.values())
    for n, (tot, cnt) in per_kernel.items():
        if cnt:
            kernels[n]["share"] = tot / total_kernel_ms
    dom = max(kernels, key=lambda n: kernels[n]["ms_per_launch"] * kernels[n]["launches"])
    pk = peaks()
    hbm = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    achieved = alg_per_launch.get(dom, 0) / (kernels[dom]["ms_per_launch"] * 1e-3) / 1e9
    roofline = {
        "kernel": dom,
        "bound": "hbm",
        "achieved": achieved,
        "peak": hbm,
        "unit": "GB/s",
        "frac": achieved / hbm,
        "peak_source": f"{pk.get('source')} (MEASURED_PEAKS.json hbm_gbs)" if pk.get("source") == "measured" else "fallback 6.65 TB/s",
        "alg_bytes_per_launch": alg_per_launch.get(dom, 0),
        "traffic": ncu_traffic(dom, args.workload),
    }

    result = {
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": wl["dtype"],
        "data": "synthetic (seeded numpy PCG64; config distributions)",
        "config": dict(native_config(wl, b, t, c, world),
                       frac_of_hbm_peak=value / world / hbm,
                       plan=dict(zip(("tma", "segments"), _capi.plan(code, b, t, c), strict=True)),
                       path=("wkv_forward + wkv_backward (backward re-runs the forward sweep)" if args.no_state
                             else "wkv_forward_with_state + wkv_backward_from_state (the autograd path)")),
        "roofline": roofline,
        "kernels": kernels,
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if not args.profile:
        result["e2e"] = run_e2e(args, wl, dev, k_np, v_np, td_np, tf_np, gy_np, tdt, world)
        # the other op pair: the schema-pure ops (the backward re-runs the forward sweep)
        other = step_state if args.no_state else step_plain
        n_other = max(5, min(args.steps, 200))
        for _ in range(3):
            other()
        _capi.timing_collect()
        _capi.timing_enable(True)
        torch.cuda.synchronize(dev)
        o0, o1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        o0.record(stream)
        for _ in range(n_other):
            other()
        o1.record(stream)
        torch.cuda.synchronize(dev)
        _capi.timing_enable(False)
        oms = max_over_ranks(o0.elapsed_time(o1), dev) / n_other
        result["state" if args.no_state else "no_state"] = {
            "value": step_bytes * world / (oms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": oms,
            "steps": n_other,
            "path": ("wkv_forward_with_state + wkv_backward_from_state" if args.no_state else
                     "wkv_forward + wkv_backward: the reference's self-contained op contract (the backward "
                     "re-runs the forward sweep); what a direct caller of the myelin:: ops gets"),
            "kernels": {n: {"ms_per_launch": tot / cnt, "launches": cnt}
                        for n, (tot, cnt) in _capi.timing_collect().items() if cnt},
        }
        if world == 1 and rank == 0:
            result["cpu_baseline"] = cpu_oracle_throughput(wl, seconds=10.0)
        if args.train_leg and "kind" not in wl:
            # the data-parallel SpikeGPT-41M train step (config 3) at this N:
            # global batch 64 over the ranks, gradients all-reduced over NCCL
            tr, tstep, *_ = measure_train(WORKLOADS["train"], steps=TRAIN_LEG_STEPS, warmup=TRAIN_LEG_WARMUP,
                                          world=world, rank=rank, dev=dev, clocks=False)
            tstep.release()
            result["train_step"] = {k: tr[k] for k in (
                "metric", "value", "unit", "ms_per_step", "allreduce", "allreduce_ms_per_step", "nccl_ranks",
                "steps", "warmup", "scaling", "loss", "gpu_launches")}
            result["train_step"].update(
                model=tr["config"]["model"], global_batch=tr["config"]["global_batch"],
                B_per_gpu=tr["config"]["B_per_gpu"], seq_len=tr["config"]["seq_len"],
                parallelism=tr["config"]["parallelism"], launch=tr["config"]["launch"],
                mfu=tr["roofline"]["frac"], mfu_peak_tflops=tr["roofline"]["peak"],
                mfu_peak_source=tr["roofline"]["peak_source"],
                tokens_per_s_per_gpu=tr["value"] / world)
        if world == 1 and rank == 0 and args.incumbent and "kind" not in wl:
            result["incumbent"] = incumbent_leg(args, wl)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_segment_sweep(args, wl):
    """One JSON line per time-segment count for the WKV op pair (saved-state
    forward + backward) on this workload: the measurement behind the plan
    choice of the C ABI (make_plan). 0 in the list means the default plan."""
    import torch

    from spikegpt_b200 import _capi

    dev = torch.device("cuda", 0)
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["dtype"]]
    code = {"bf16": _capi.DTYPE_BF16, "fp16": _capi.DTYPE_F16, "fp32": _capi.DTYPE_F32}[wl["dtype"]]
    b, t, c = wl["B"], wl["T"], wl["C"]
    k_np, v_np, td_np, tf_np, gy_np = make_inputs(wl, seed=0)
    k, v, gy = (torch.as_tensor(x).to(dev, tdt) for x in (k_np, v_np, gy_np))
    td, tf = torch.as_tensor(td_np).to(dev), torch.as_tensor(tf_np).to(dev)
    w = -torch.exp(td)
    y, gk, gv = torch.empty_like(k), torch.empty_like(k), torch.empty_like(k)
    gtd, gtf = torch.empty_like(td), torch.empty_like(td)
    lib = _capi.lib()
    sp = torch.cuda.current_stream(dev).cuda_stream
    step_bytes = BYTES_PER_ELEM[wl["dtype"]] * b * t * c
    for nseg in [int(x) for x in args.sweep_segments.split(",")]:
        _capi.set_debug_overrides(force_segments=nseg)
        try:
            fws_n = int(lib.wkv_forward_workspace_size(code, b, t, c))
            bws_n = int(lib.wkv_backward_workspace_size(code, b, t, c))
            st_n = int(lib.wkv_state_size(code, b, t, c))
            fws = torch.empty(max(fws_n, 1), dtype=torch.uint8, device=dev)
            bws = torch.empty(max(bws_n, 1), dtype=torch.uint8, device=dev)
            state = torch.empty(max(st_n, 16), dtype=torch.uint8, device=dev)
            plan = _capi.plan(code, b, t, c)

            def step():
                _capi.check(lib.wkv_forward_with_state(code, k.data_ptr(), v.data_ptr(), td.data_ptr(),
                                                       tf.data_ptr(), y.data_ptr(), state.data_ptr(), st_n, b, t,
                                                       c, fws.data_ptr(), fws_n, sp), "wkv_forward_with_state")
                _capi.check(lib.wkv_backward_from_state(code, gy.data_ptr(), w.data_ptr(), tf.data_ptr(),
                                                        k.data_ptr(), v.data_ptr(), state.data_ptr(), st_n,
                                                        gk.data_ptr(), gv.data_ptr(), gtd.data_ptr(),
                                                        gtf.data_ptr(), b, t, c, bws.data_ptr(), bws_n, sp),
                            "wkv_backward_from_state")

            for _ in range(max(3, args.warmup)):
                step()
            torch.cuda.synchronize(dev)
            _capi.timing_collect()
            _capi.timing_enable(True)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                step()
            e1.record()
            torch.cuda.synchronize(dev)
            _capi.timing_enable(False)
            ms = e0.elapsed_time(e1) / args.steps
            kernels = {n: round(tot / cnt * 1e3, 2) for n, (tot, cnt) in _capi.timing_collect().items() if cnt}
        finally:
            _capi.set_debug_overrides()
        print(json.dumps({"workload": args.workload, "B": b, "T": t, "C": c, "forced_segments": nseg,
                          "plan": {"tma": bool(plan[0]), "segments": int(plan[1])}, "ms_per_step": ms,
                          "GB_s": step_bytes / (ms * 1e-3) / 1e9, "us_per_launch": kernels}), flush=True)


def run_step(args, wl):
    """The recurrent step (generation): one wkv_step launch per step over B
    streams, state resident on the device and updated in place, new k, v each
    step (the same buffers, as a decode loop refills them). Algorithmic bytes
    per element: read k, v and the three state planes, write y and the state."""
    import torch
    import torch.distributed as dist

    from spikegpt_b200 import _capi

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    from spikegpt_b200.sharding import max_over_ranks

    tk = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["dtype"]]
    ts = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["state"]]
    ck = {"bf16": _capi.DTYPE_BF16, "fp16": _capi.DTYPE_F16, "fp32": _capi.DTYPE_F32}[wl["dtype"]]
    cs = {"bf16": _capi.DTYPE_BF16, "fp16": _capi.DTYPE_F16, "fp32": _capi.DTYPE_F32}[wl["state"]]
    b, c = wl["B"], wl["C"]
    rng = np.random.default_rng(rank)
    k = torch.as_tensor((rng.standard_normal((b, c)) * wl["kscale"]).astype(np.float32)).to(dev, tk)
    v = torch.as_tensor(rng.standard_normal((b, c)).astype(np.float32)).to(dev, tk)
    td = torch.as_tensor(rng.uniform(-5, 1, c).astype(np.float32)).to(dev)
    tf = torch.as_tensor(rng.uniform(-1, 1, c).astype(np.float32)).to(dev)
    num = torch.zeros((b, c), device=dev, dtype=ts)
    den = torch.zeros_like(num)
    ls = torch.full((b, c), torch.finfo(ts).min, device=dev, dtype=ts)
    y = torch.empty_like(num)
    lib = _capi.lib()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream

    def step(kk=k, vv=v):
        _capi.check(lib.wkv_step(ck, cs, kk.data_ptr(), vv.data_ptr(), td.data_ptr(), tf.data_ptr(), num.data_ptr(),
                                 den.data_ptr(), ls.data_ptr(), y.data_ptr(), b, c, sp), "wkv_step")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    sampler = None if args.profile else ClockSampler(local)
    time.sleep(0.3 if sampler else 0)
    _capi.timing_collect()
    _capi.timing_enable(True)
    launches0 = sum(_capi.launch_counts().values())
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    host1 = time.time()
    if world > 1:
        dist.barrier(device_ids=[local])
    _capi.timing_enable(False)
    launches = sum(_capi.launch_counts().values()) - launches0
    per_kernel = _capi.timing_collect()
    ms = max_over_ranks(ev0.elapsed_time(ev1), dev)
    if sampler:
        time.sleep(0.25)
        sampler.stop()
    clocks = sampler.summary(host0, host1) if sampler else None

    per_elem = 2 * STEP_BYTES[wl["dtype"]] + 7 * STEP_BYTES[wl["state"]]
    step_bytes = per_elem * b * c
    value = step_bytes * args.steps * world / (ms * 1e-3) / 1e9
    tot, cnt = per_kernel["wkv_step_kernel"]
    pk = peaks()
    hbm = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    achieved = step_bytes / (tot / cnt * 1e-3) / 1e9
    result = {
        "metric": STEP_METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms / args.steps,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": wl["dtype"],
        "data": "synthetic (seeded numpy PCG64)",
        "config": {
            "workload": wl["desc"], "B_per_gpu": b, "C": c, "state_dtype": wl["state"],
            "tokens_per_s": b * args.steps * world / (ms * 1e-3),
            "parallelism": f"{world} stream-sharded replica(s), no collective",
            "l2": f"{step_bytes / 1e6:.0f} MB moved per step (> L2); no flush",
        },
        "roofline": {"kernel": "wkv_step_kernel", "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "alg_bytes_per_launch": step_bytes,
                     "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if pk.get("source") == "measured"
                     else "fallback 6.65 TB/s",
                     "traffic": ncu_traffic("wkv_step_kernel", args.workload)},
        "kernels": {"wkv_step_kernel": {"ms_per_launch": tot / cnt, "launches": cnt, "share": 1.0}},
        "gpu_launches": int(launches),
        "clocks": clocks,
    }
    if not args.profile:
        # e2e: each step's k, v from pinned host memory, y back to the host;
        # the state stays on the device (a decode loop keeps it there)
        hk, hv = k.cpu().pin_memory(), v.cpu().pin_memory()
        hy = torch.empty(y.shape, dtype=y.dtype).pin_memory()
        dk, dv = torch.empty_like(k), torch.empty_like(v)

        def e2e_step():
            dk.copy_(hk, non_blocking=True)
            dv.copy_(hv, non_blocking=True)
            step(dk, dv)
            hy.copy_(y, non_blocking=True)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize(dev)
        ems = max_over_ranks(e0.elapsed_time(e1), dev)
        result["e2e"] = {"value": step_bytes * args.e2e_steps * world / (ems * 1e-3) / 1e9, "unit": "GB/s",
                         "h2d_bytes_per_step": 2 * hk.numel() * hk.element_size(),
                         "d2h_bytes_per_step": hy.numel() * hy.element_size(),
                         "steps": args.e2e_steps, "ms_per_step": ems / args.e2e_steps,
                         "path": "wkv_step through the C ABI; k, v copied in and y copied out every step"}
        if world == 1 and rank == 0:
            result["cpu_baseline"] = cpu_step_throughput(wl)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_lif(args, wl):
    """LIF sequence op: one lif_forward (keeping its membrane state) plus one
    lif_backward per step through the C ABI on device-resident inputs.
    Algorithmic bytes per element: forward x in, spikes out; backward grad,
    x in, grad x out (5 x the element size)."""
    import torch
    import torch.distributed as dist

    from spikegpt_b200 import _capi, surrogate_lif
    from spikegpt_b200.sharding import max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    tdt = {"bf16": torch.bfloat16, "fp16": torch.float16, "fp32": torch.float32}[wl["dtype"]]
    code = {"bf16": _capi.DTYPE_BF16, "fp16": _capi.DTYPE_F16, "fp32": _capi.DTYPE_F32}[wl["dtype"]]
    b, t, c = wl["B"], wl["T"], wl["C"]
    rng = np.random.default_rng(rank)
    x_np = (rng.standard_normal((b, t, c)) * wl["kscale"] + 0.3).astype(np.float32)
    gs_np = rng.standard_normal((b, t, c)).astype(np.float32)
    x = torch.as_tensor(x_np).to(dev, tdt)
    gs = torch.as_tensor(gs_np).to(dev, tdt)
    spikes, gx = torch.empty_like(x), torch.empty_like(x)
    lib = _capi.lib()
    nst = int(lib.lif_state_size(code, b, t, c))
    state = torch.empty(nst // 4, dtype=torch.float32, device=dev)
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    prm = (2.0, 1.0, 0.0, 2.0)  # tau, threshold, reset, surrogate_slope (the reference's defaults)

    def step():
        _capi.check(lib.lif_forward(code, x.data_ptr(), spikes.data_ptr(), state.data_ptr(), nst, b, t, c, *prm, sp),
                    "lif_forward")
        _capi.check(lib.lif_backward(code, gs.data_ptr(), x.data_ptr(), state.data_ptr(), nst, gx.data_ptr(),
                                     b, t, c, *prm, sp), "lif_backward")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    sampler = None if args.profile else ClockSampler(local)
    time.sleep(0.3 if sampler else 0)
    _capi.timing_collect()
    _capi.timing_enable(True)
    launches0 = sum(_capi.launch_counts().values())
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    host1 = time.time()
    if world > 1:
        dist.barrier(device_ids=[local])
    _capi.timing_enable(False)
    launches = sum(_capi.launch_counts().values()) - launches0
    per_kernel = _capi.timing_collect()
    ms = max_over_ranks(ev0.elapsed_time(ev1), dev)
    if sampler:
        time.sleep(0.25)
        sampler.stop()
    clocks = sampler.summary(host0, host1) if sampler else None
    es = STEP_BYTES[wl["dtype"]]
    elems = b * t * c
    value = 5 * es * elems * args.steps * world / (ms * 1e-3) / 1e9
    alg = {"lif_fwd_kernel": 2 * es * elems, "lif_bwd_kernel": 3 * es * elems}
    kernels = {n: {"ms_per_launch": tot / cnt, "launches": cnt} for n, (tot, cnt) in per_kernel.items() if cnt}
    total = sum(k["ms_per_launch"] * k["launches"] for k in kernels.values())
    for k in kernels.values():
        k["share"] = k["ms_per_launch"] * k["launches"] / total
    dom = max(kernels, key=lambda n: kernels[n]["share"])
    pk = peaks()
    hbm = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    achieved = alg[dom] / (kernels[dom]["ms_per_launch"] * 1e-3) / 1e9
    result = {
        "metric": LIF_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": wl["dtype"], "data": "synthetic (seeded numpy PCG64)",
        "config": {"workload": wl["desc"], "B_per_gpu": b, "T": t, "C": c,
                   "parallelism": f"{world} batch-sharded replica(s), no collective",
                   "l2": f"{4 * es * elems / 1e6:.0f} MB of inputs read per step (> L2); no flush"},
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s",
                     "frac": achieved / hbm, "alg_bytes_per_launch": alg[dom],
                     "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if pk.get("source") == "measured"
                     else "fallback 6.65 TB/s",
                     "traffic": ncu_traffic(dom, args.workload)},
        "kernels": kernels, "gpu_launches": int(launches), "clocks": clocks,
    }
    if not args.profile:
        hx = torch.as_tensor(x_np).to(tdt).pin_memory()
        hgs = torch.as_tensor(gs_np).to(tdt).pin_memory()
        hs, hgx = torch.empty_like(hx).pin_memory(), torch.empty_like(hx).pin_memory()

        def e2e_step():
            xd = hx.to(dev, non_blocking=True).requires_grad_()
            out = surrogate_lif(xd)
            out.backward(hgs.to(dev, non_blocking=True))
            hs.copy_(out.detach(), non_blocking=True)
            hgx.copy_(xd.grad, non_blocking=True)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize(dev)
        ems = max_over_ranks(e0.elapsed_time(e1), dev)
        result["e2e"] = {"value": 5 * es * elems * args.e2e_steps * world / (ems * 1e-3) / 1e9, "unit": "GB/s",
                         "h2d_bytes_per_step": 2 * es * elems, "d2h_bytes_per_step": 2 * es * elems,
                         "steps": args.e2e_steps, "ms_per_step": ems / args.e2e_steps,
                         "path": "autograd through spikegpt_b200.surrogate_lif, pinned host buffers"}
        if world == 1 and rank == 0:
            result["cpu_baseline"] = cpu_lif_throughput(wl)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def run_rwkv7(args, wl):
    """RWKV-7 DPLR forward: one rwkv7_forward per step through the C ABI on
    device-resident inputs. Algorithmic bytes per element: r, w, k, v, a, b in
    and y out, 7 x 4 B (the per-head state stays on chip)."""
    import torch
    import torch.distributed as dist

    from spikegpt_b200 import _capi
    from spikegpt_b200.rwkv7 import HEAD_SIZE, dplr_inputs, rwkv7_forward_op
    from spikegpt_b200.sharding import max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=dev)
    b, t, h = wl["B"], wl["T"], wl["H"]
    host = dplr_inputs(b, t, h, seed=rank)
    ins = [x.to(dev) for x in host]
    y = torch.empty_like(ins[0])
    s_out = torch.empty((b, h, HEAD_SIZE, HEAD_SIZE), dtype=torch.float32, device=dev)
    lib = _capi.lib()
    stream = torch.cuda.current_stream(dev)
    sp = stream.cuda_stream
    ptrs = [x.data_ptr() for x in ins]

    def step():
        _capi.check(lib.rwkv7_forward(*ptrs, None, y.data_ptr(), s_out.data_ptr(), b, t, h, HEAD_SIZE, sp),
                    "rwkv7_forward")

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize(dev)
    sampler = None if args.profile else ClockSampler(local)
    time.sleep(0.3 if sampler else 0)
    _capi.timing_collect()
    _capi.timing_enable(True)
    launches0 = sum(_capi.launch_counts().values())
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize(dev)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host0 = time.time()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize(dev)
    host1 = time.time()
    if world > 1:
        dist.barrier(device_ids=[local])
    _capi.timing_enable(False)
    launches = sum(_capi.launch_counts().values()) - launches0
    per_kernel = _capi.timing_collect()
    ms = max_over_ranks(ev0.elapsed_time(ev1), dev)
    if sampler:
        time.sleep(0.25)
        sampler.stop()
    clocks = sampler.summary(host0, host1) if sampler else None
    elems = b * t * h * HEAD_SIZE
    alg = 7 * 4 * elems
    value = alg * args.steps * world / (ms * 1e-3) / 1e9
    tot, cnt = per_kernel["rwkv7_fwd_kernel"]
    pk = peaks()
    hbm = float(pk.get("hbm_gbs", PEAKS_FALLBACK["hbm_gbs"]))
    achieved = alg / (tot / cnt * 1e-3) / 1e9
    result = {
        "metric": RWKV7_METRIC, "value": value, "unit": "GB/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms / args.steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "fp32", "data": "synthetic (seeded torch; rwkv7.dplr_inputs)",
        "tokens_per_s": b * t * args.steps * world / (ms * 1e-3),
        "config": {"workload": wl["desc"], "B_per_gpu": b, "T": t, "H": h, "head_size": HEAD_SIZE,
                   "parallelism": f"{world} batch-sharded replica(s), no collective",
                   "l2": f"{alg / 1e6:.0f} MB moved per step (> L2); no flush",
                   "form": "sequential over T on CUDA cores (the chunked tensor-core form is not built)"},
        "roofline": {"kernel": "rwkv7_fwd_kernel", "bound": "hbm", "achieved": achieved, "peak": hbm,
                     "unit": "GB/s", "frac": achieved / hbm, "alg_bytes_per_launch": alg,
                     "peak_source": "measured (MEASURED_PEAKS.json hbm_gbs)" if pk.get("source") == "measured"
                     else "fallback 6.65 TB/s", "traffic": ncu_traffic("rwkv7_fwd_kernel", args.workload)},
        "gpu_launches": int(launches), "clocks": clocks,
    }
    if not args.profile:
        pins = [x.pin_memory() for x in host]
        hy = torch.empty_like(pins[0]).pin_memory()

        def e2e_step():
            yd, _ = rwkv7_forward_op(*(x.to(dev, non_blocking=True) for x in pins))
            hy.copy_(yd, non_blocking=True)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(args.e2e_steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize(dev)
        ems = max_over_ranks(e0.elapsed_time(e1), dev)
        result["e2e"] = {"value": alg * args.e2e_steps * world / (ems * 1e-3) / 1e9, "unit": "GB/s",
                         "h2d_bytes_per_step": 6 * 4 * elems, "d2h_bytes_per_step": 4 * elems,
                         "steps": args.e2e_steps, "ms_per_step": ems / args.e2e_steps,
                         "path": "spikegpt_b200.rwkv7.rwkv7_forward_op, pinned host buffers"}
        if world == 1 and rank == 0:
            result["cpu_baseline"] = cpu_rwkv7_throughput(wl)
    if rank == 0:
        print(json.dumps(result), flush=True)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def cpu_rwkv7_throughput(wl: dict, seconds: float = 3.0):
    """The float64 numpy restatement (oracle) on one sequence of the workload."""
    from oracle import oracle
    from spikegpt_b200.rwkv7 import HEAD_SIZE, dplr_inputs

    ins = [x.numpy() for x in dplr_inputs(1, wl["T"], wl["H"], seed=0)]
    n, t0 = 0, time.perf_counter()
    while True:
        oracle.rwkv7_forward_numpy(*ins)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    return {"value": 7 * 4 * wl["T"] * wl["H"] * HEAD_SIZE * n / dt / 1e9, "unit": "GB/s", "cores": 1,
            "kind": "port", "sample": f"{n} x (1 of {wl['B']} sequences, T={wl['T']}, H={wl['H']}), numpy float64",
            "note": "the reference has no RWKV-7 code; the oracle restates the published recurrence"}


def run_rwkv7_reference(args, wl):
    """Reference arm of the RWKV-7 workload: the reference ships no
    implementation, so the arm times the oracle restatement on the host."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    base = cpu_rwkv7_throughput(wl, seconds=2.0)
    print(json.dumps({"metric": RWKV7_METRIC, "value": base["value"], "unit": "GB/s",
                      "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps,
                      "warmup": args.warmup, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
                      "dtype": "fp32", "data": "synthetic", "config": {"workload": wl["desc"]},
                      "impl": "reference", "cpu_baseline": base,
                      "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0,
                              "d2h_bytes_per_step": 0}}), flush=True)


def cpu_lif_throughput(wl: dict, seconds: float = 5.0):
    """The float32 LIF oracle fwd+bwd (a single-threaded C loop) on one batch row."""
    from oracle import oracle

    rng = np.random.default_rng(0)
    x = (rng.standard_normal((1, wl["T"], wl["C"])) * wl["kscale"] + 0.3).astype(np.float32)
    gs = rng.standard_normal(x.shape).astype(np.float32)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        oracle.lif_forward(x, dtype=np.float32)
        oracle.lif_backward(gs, x, dtype=np.float32)
        n += 1
    el = time.perf_counter() - t0
    return {"value": 5 * STEP_BYTES[wl["dtype"]] * x.size * n / el / 1e9, "unit": "GB/s", "cores": 1,
            "kind": "port", "sample": f"{n} x (1 of {wl['B']} batch rows), float32, {el:.1f} s",
            "host_cpus": os.cpu_count()}


def cpu_step_throughput(wl: dict, seconds: float = 5.0):
    """The float32 oracle step (a single-threaded C loop) on 64 of the
    workload's streams, repeated for about `seconds`."""
    from oracle import oracle

    b, c = 64, wl["C"]
    rng = np.random.default_rng(0)
    k = (rng.standard_normal((b, c)) * wl["kscale"]).astype(np.float32)
    v = rng.standard_normal((b, c)).astype(np.float32)
    td = rng.uniform(-5, 1, c).astype(np.float32)
    tf = rng.uniform(-1, 1, c).astype(np.float32)
    state = oracle.initial_step_state(b, c, np.float32)
    n, t0 = 0, time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        _, *state = oracle.step(k, v, td, tf, *state, dtype=np.float32)
        n += 1
    el = time.perf_counter() - t0
    per_elem = 2 * STEP_BYTES[wl["dtype"]] + 7 * STEP_BYTES[wl["state"]]
    return {"value": per_elem * b * c * n / el / 1e9, "unit": "GB/s", "cores": 1, "kind": "port",
            "sample": f"{n} steps of 64 streams x C={c}, float32, {el:.1f} s", "host_cpus": os.cpu_count()}


def ncu_traffic(kernel: str, workload: str):
    """DRAM bytes per launch of `kernel` from the committed ncu summary for the
    workload (profiles/*.md line 'dram_bytes_per_launch[<kernel>] = N'), else None."""
    pat = re.compile(r"dram_bytes_per_launch\[" + re.escape(kernel) + r"\]\[" + re.escape(workload) + r"\]\s*=\s*([0-9.eE+]+)")
    for p in sorted((ROOT / "profiles").glob("*.md")):
        m = pat.search(p.read_text())
        if m:
            return float(m.group(1))
    return None


def run_e2e(args, wl, dev, k_np, v_np, td_np, tf_np, gy_np, tdt, world):
    """The metric through the public autograd op with host buffers (pinned).

    Each step moves that step's k, v, grad_y host->device and y, grad_key,
    grad_value, grad_time_decay, grad_time_first device->host, as a user with
    host-resident data does. Copies in, compute and copies out run on three
    CUDA streams ordered by events, so one step's results travel to the host
    while the next step's inputs travel to the device (the two PCIe directions
    overlap). --e2e-chunks > 1 also splits each step's batch into chunks
    (batch rows are independent; the per-channel gradients accumulate across
    chunks in the leaves' .grad, as autograd does for any split batch).
    """
    import torch
    import torch.distributed as dist

    import spikegpt_b200  # noqa: F401
    from spikegpt_b200 import weighted_key_value_triton_bf16io

    def pin(x, dt):
        return torch.as_tensor(x).to(dt).pin_memory()

    hk, hv, hgy = pin(k_np, tdt), pin(v_np, tdt), pin(gy_np, tdt)
    htd, htf = pin(td_np, torch.float32), pin(tf_np, torch.float32)
    hy, hgk, hgv = (torch.empty_like(hk).pin_memory() for _ in range(3))
    hgtd, hgtf = torch.empty_like(htd).pin_memory(), torch.empty_like(htf).pin_memory()
    h2d = sum(x.numel() * x.element_size() for x in (hk, hv, hgy, htd, htf))
    d2h = sum(x.numel() * x.element_size() for x in (hy, hgk, hgv, hgtd, hgtf))

    b = wl["B"]
    nch = max(1, min(args.e2e_chunks, b))
    bounds = [(i * b // nch, (i + 1) * b // nch) for i in range(nch)]
    s_in, s_comp, s_out = torch.cuda.Stream(dev), torch.cuda.Stream(dev), torch.cuda.Stream(dev)
    # device input slots, one per chunk
    dk = [torch.empty((hi - lo,) + tuple(hk.shape[1:]), dtype=tdt, device=dev) for lo, hi in bounds]
    dv = [torch.empty_like(x) for x in dk]
    dgy = [torch.empty_like(x) for x in dk]
    dtd = torch.empty(htd.shape, dtype=torch.float32, device=dev)
    dtf = torch.empty_like(dtd)
    slot_free = [torch.cuda.Event() for _ in bounds]  # compute of the slot's last use is done
    for e in slot_free:
        e.record(s_comp)

    def step():
        ev_par = torch.cuda.Event()
        with torch.cuda.stream(s_in):
            s_in.wait_event(slot_free[-1])  # the previous step's compute no longer reads dtd, dtf
            dtd.copy_(htd, non_blocking=True)
            dtf.copy_(htf, non_blocking=True)
            ev_par.record(s_in)
        with torch.cuda.stream(s_comp):
            s_comp.wait_event(ev_par)
            td = dtd.detach().requires_grad_()
            tf = dtf.detach().requires_grad_()
        for i, (lo, hi) in enumerate(bounds):
            ev_in = torch.cuda.Event()
            with torch.cuda.stream(s_in):
                s_in.wait_event(slot_free[i])
                dk[i].copy_(hk[lo:hi], non_blocking=True)
                dv[i].copy_(hv[lo:hi], non_blocking=True)
                dgy[i].copy_(hgy[lo:hi], non_blocking=True)
                ev_in.record(s_in)
            with torch.cuda.stream(s_comp):
                s_comp.wait_event(ev_in)
                k = dk[i].detach().requires_grad_()
                v = dv[i].detach().requires_grad_()
                y = weighted_key_value_triton_bf16io(k, v, td, tf)
                y.backward(dgy[i])
                ev_done = torch.cuda.Event()
                ev_done.record(s_comp)
                slot_free[i] = ev_done
            with torch.cuda.stream(s_out):
                s_out.wait_event(ev_done)
                for src, dst in ((y.detach(), hy[lo:hi]), (k.grad, hgk[lo:hi]), (v.grad, hgv[lo:hi])):
                    dst.copy_(src, non_blocking=True)
                    src.record_stream(s_out)  # not reused by the allocator before the copy ends
        with torch.cuda.stream(s_out):
            s_out.wait_stream(s_comp)
            for src, dst in ((td.grad, hgtd), (tf.grad, hgtf)):
                dst.copy_(src, non_blocking=True)
                src.record_stream(s_out)
        torch.cuda.current_stream(dev).wait_stream(s_out)

    for _ in range(3):
        step()
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.e2e_steps):
        step()
    e1.record()
    torch.cuda.synchronize(dev)
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    elems = wl["B"] * wl["T"] * wl["C"]
    value = BYTES_PER_ELEM[wl["dtype"]] * elems * args.e2e_steps * world / (ms * 1e-3) / 1e9
    return {"value": value, "unit": "GB/s", "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
            "steps": args.e2e_steps, "ms_per_step": ms / args.e2e_steps, "chunks": nch,
            "path": "autograd through spikegpt_b200.weighted_key_value_triton_bf16io (myelin::wkv_forward_bf16io) "
                    "on batch chunks; pinned host buffers; copy-in, compute and copy-out streams overlapped"}


# ----------------------------------------------------------- reference arm


def run_reference(args, wl):
    """Reference arm: the reference's own CPU WKV path on the host cores
    (weighted_key_value, rank 0 only), or the C restatement of its arithmetic
    (oracle/wkv_oracle.c) when the reference is not installed."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if reference_available():
        base = reference_cpu_throughput(wl, steps=args.steps, warmup=args.warmup)
        note = ("the reference's own CPU implementation of the path: weighted_key_value "
                "(src/spikegpt/language.py:452-527) from baseline/_ref, fp32, torch threads = host cores")
    else:
        base = cpu_oracle_throughput(wl, steps=args.steps, warmup=args.warmup)
        note = ("baseline/_ref absent: the C restatement of the reference's WKV arithmetic "
                "(oracle/wkv_oracle.c), float32, on the host cores")
    b, t, c = wl["B"], wl["T"], wl["C"]
    out = {
        "metric": METRIC,
        "value": base["value"],
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": wl["dtype"],
        "data": "synthetic (seeded numpy PCG64; config distributions)",
        "config": native_config(wl, b, t, c, world),
        "impl": "reference",
        "cpu_baseline": base,
        "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": note,
    }
    print(json.dumps(out), flush=True)


def run_step_reference(args, wl):
    """Reference arm of the step workload: the oracle step on the host, rank 0."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    base = cpu_step_throughput(wl, seconds=2.0)
    out = {"metric": STEP_METRIC, "value": base["value"], "unit": "GB/s",
           "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": wl["dtype"],
           "data": "synthetic (seeded numpy PCG64)", "config": {"workload": wl["desc"], "C": wl["C"]},
           "impl": "reference", "cpu_baseline": base,
           "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference's step is PyTorch code inside SpikeTimeMix.step; this arm times the C "
                   "restatement of its arithmetic (oracle/wkv_oracle.c) on the host"}
    print(json.dumps(out), flush=True)


def run_lif_reference(args, wl):
    """Reference arm of the LIF workload: the oracle on the host, rank 0."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    base = cpu_lif_throughput(wl, seconds=2.0)
    out = {"metric": LIF_METRIC, "value": base["value"], "unit": "GB/s",
           "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
           "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": wl["dtype"],
           "data": "synthetic (seeded numpy PCG64)", "config": {"workload": wl["desc"]},
           "impl": "reference", "cpu_baseline": base,
           "e2e": {"value": base["value"], "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
           "note": "the reference's CPU path is its per-step PyTorch loop; this arm times the C restatement "
                   "of that loop (oracle/wkv_oracle.c) on the host"}
    print(json.dumps(out), flush=True)


def zipf_tokens(rng, shape, vocab: int, s: float):
    """iid token ids with P(rank r) proportional to r^-s over the vocabulary
    (rank r -> id r - 1)."""
    w = np.arange(1, vocab + 1, dtype=np.float64) ** -s
    return rng.choice(vocab, size=shape, p=w / w.sum()).astype(np.int64)


def train_kernel_split(model, opt, x, y, dev, top: int) -> None:
    """Per-kernel device time of the train step: two eager steps (the same
    kernels a graph replay runs) under the torch profiler's CUDA activity,
    averaged per step, printed to stderr."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    from spikegpt_b200.train import TrainStep

    step = TrainStep(model, opt, tuple(x.shape), device=dev, graph=False)
    for _ in range(2):
        step(x, y)
    torch.cuda.synchronize(dev)
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(2):
            step(x, y)
        torch.cuda.synchronize(dev)
    rows = sorted(((e.device_time_total, e.count, e.key) for e in prof.key_averages() if e.device_time_total > 0),
                  reverse=True)
    total = sum(r[0] for r in rows)
    print(f"device time per step {total / 2e3:.2f} ms over {sum(r[1] for r in rows) // 2} kernels "
          f"(batch {x.shape[0]} x {x.shape[1]})", file=sys.stderr)
    for t_us, n, key in rows[:top]:
        print(f"  {t_us / 2e3:8.3f} ms {n // 2:5d}  {key[:110]}", file=sys.stderr)


def measure_train(wl, *, steps: int, warmup: int, world: int, rank: int, dev, global_batch=None,
                  eager: bool = False, clocks: bool = True, e2e_steps: int = 0, overlap: bool = False,
                  micro_batches: int | None = None):
    """Time the data-parallel train step (the process group, if any, is already
    initialized). Returns (result dict, TrainStep, model, optimizer, x, y); the
    caller releases the step before destroying the process group."""
    import torch

    from spikegpt_b200 import _capi
    from spikegpt_b200.model import SPIKEGPT_41M, SPIKEGPT_216M, SpikeGPT, flops_per_token
    from spikegpt_b200.sharding import max_over_ranks
    from spikegpt_b200.train import TrainStep

    import torch.distributed as dist

    cfg = {"41m": SPIKEGPT_41M, "216m": SPIKEGPT_216M}[wl["model"]]
    gb, t = global_batch or wl["global_batch"], wl["T"]
    if gb % world:
        raise SystemExit(f"global batch {gb} does not split over {world} ranks")
    b = gb // world
    torch.manual_seed(0)
    model = SpikeGPT(cfg).to(dev)
    opt = torch.optim.AdamW(model.parameters(), lr=6e-4, weight_decay=0.1, fused=True)
    rng = np.random.default_rng(rank)
    ids_np = zipf_tokens(rng, (b, t + 1), cfg.vocab_size, wl["zipf"])
    ids = torch.as_tensor(ids_np).to(dev)
    x, y = ids[:, :-1].contiguous(), ids[:, 1:].contiguous()
    launches_before = sum(_capi.launch_counts().values())
    if micro_batches is None:  # measured (SpikeGPT-41M, one B200): two micro-batches pay at 8 and 16 sequences
        micro_batches = 2 if 8 <= b <= 16 and not overlap else 1
    step = TrainStep(model, opt, (b, t), device=dev, graph=not eager, overlap=overlap, micro_batches=micro_batches)
    capture_launches = sum(_capi.launch_counts().values()) - launches_before

    for _ in range(warmup):
        loss = step(x, y)
    torch.cuda.synchronize(dev)
    local = dev.index or 0
    sampler = ClockSampler(local) if clocks else None
    time.sleep(0.3 if sampler else 0)
    launches0 = sum(_capi.launch_counts().values())
    if world > 1:
        dist.barrier(device_ids=[local])
    torch.cuda.synchronize(dev)
    step.time_allreduce(world > 1)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    host0 = time.time()
    ev0.record()
    for _ in range(steps):
        loss = step(x, y)
    ev1.record()
    torch.cuda.synchronize(dev)
    host1 = time.time()
    ar_ms, ar_n = step.allreduce_ms()
    step.time_allreduce(False)
    if world > 1:
        dist.barrier(device_ids=[local])
    # eager launches go through the C ABI's counters; a graph replay runs the
    # kernels counted while it was captured
    launches = sum(_capi.launch_counts().values()) - launches0 + steps * step.captured_launches
    ms = max_over_ranks(ev0.elapsed_time(ev1), dev)
    ar = max_over_ranks(ar_ms / ar_n if ar_n else 0.0, dev)
    if sampler:
        time.sleep(0.25)
        sampler.stop()
    tokens = gb * t * steps
    value = tokens / (ms * 1e-3)
    fpt = flops_per_token(cfg)
    pk = peaks()
    peak = float(pk.get("bf16_tflops_sustained", pk.get("bf16_tflops", PEAKS_FALLBACK_TFLOPS)))
    achieved = value * fpt / world / 1e12
    name = {"41m": "SpikeGPT-41M", "216m": "SpikeGPT-216M"}[wl["model"]]
    result = {
        "metric": TRAIN_METRICS[wl["model"]], "value": value, "unit": "tokens/s", "n_gpus": world,
        "steps": steps, "warmup": warmup, "ms_per_step": ms / steps, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": f"synthetic Zipf({wl['zipf']}) token ids, seeded numpy PCG64 per rank",
        "config": {"workload": wl["desc"], "model": name, "global_batch": gb, "seq_len": t, "B_per_gpu": b,
                   "params": sum(p.numel() for p in model.parameters()),
                   "parallelism": f"dp{world}" + ((" (bucketed NCCL all-reduce, AVG)" if step.overlap else
                                                   " (one NCCL all-reduce, AVG)") if world > 1 else ""),
                   "launch": "eager" if eager else "CUDA graph (forward + backward), eager all-reduce "
                                                   "and fused AdamW",
                   "weights": ("bf16 copies cast once a step, weight gradients on a side stream"
                               if step.cache is not None else "autocast casts"),
                   "micro_batches": step.micro,
                   "l2": "model state and activations far above L2; no flush"},
        "allreduce_ms_per_step": ar if world > 1 and not step.overlap else None,
        "allreduce": (f"{len(step.buckets)} buckets of about 25 MB, all-reduced asynchronously during the backward "
                      "(captured in the graph)" if step.overlap else
                      "one all-reduce of the flat gradients after the backward" if world > 1 else "none (one rank)"),
        "nccl_ranks": world if world > 1 else 0,
        "roofline": {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                     "frac": achieved / peak, "flops_per_token": fpt,
                     "peak_source": "measured sustained (MEASURED_PEAKS.json bf16_tflops_sustained)"
                     if pk.get("source") == "measured" else "fallback 1.59 PFLOP/s", "traffic": None,
                     "note": "model FLOPs utilisation (6 x matmul weights per token) per GPU"},
        "loss": float(loss.item()), "gpu_launches": int(launches),
        "clocks": sampler.summary(host0, host1) if sampler else None,
        "graph_capture_launches": int(capture_launches),
    }
    if e2e_steps:
        hx = torch.as_tensor(ids_np).pin_memory()

        def e2e_step():
            d = hx.to(dev, non_blocking=True)
            return step(d[:, :-1], d[:, 1:]).to("cpu", non_blocking=True)

        for _ in range(3):
            e2e_step()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(e2e_steps):
            e2e_step()
        e1.record()
        torch.cuda.synchronize(dev)
        ems = max_over_ranks(e0.elapsed_time(e1), dev)
        result["e2e"] = {"value": gb * t * e2e_steps / (ems * 1e-3), "unit": "tokens/s",
                         "h2d_bytes_per_step": int(hx.numel() * 8), "d2h_bytes_per_step": 4,
                         "steps": e2e_steps, "ms_per_step": ems / e2e_steps,
                         "path": "token ids copied from pinned host memory each step, loss read back"}
    return result, step, model, opt, x, y


def run_train(args, wl):
    """Data-parallel train step of SpikeGPT (this package's model and ops): the
    global batch split over the ranks (per-rank work shrinks as ranks grow:
    strong scaling), bf16 autocast, fused AdamW with weight decay 0.1. A step
    is forward, backward, the gradient all-reduce (NCCL, N > 1) and the
    optimizer step on resident synthetic tokens; forward and backward replay
    one CUDA graph (``spikegpt_b200.train.TrainStep``) unless --eager."""
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        dist.init_process_group("nccl", timeout=timedelta(seconds=180), device_id=dev)
    result, step, model, opt, x, y = measure_train(
        wl, steps=args.steps, warmup=args.warmup, world=world, rank=rank, dev=dev,
        global_batch=args.global_batch, eager=args.eager, clocks=not args.profile,
        e2e_steps=0 if args.profile else args.e2e_steps, overlap=args.overlap, micro_batches=args.micro_batches)
    result["cpu_baseline"] = None
    result["cpu_baseline_note"] = ("no CPU leg: the model step runs only on this package's CUDA ops, and the "
                                   "reference's own CPU step needs myelin@68b8ebb, absent")
    if rank == 0:
        print(json.dumps(result), flush=True)
    step.release()
    if args.kernel_split and rank == 0:
        train_kernel_split(model, opt, x, y, dev, args.kernel_split)
    if world > 1:
        dist.barrier(device_ids=[local])
        dist.destroy_process_group()


def main():
    args = parse_args()
    wl = WORKLOADS[args.workload]
    if wl.get("kind") == "train":
        if args.impl == "reference":
            if int(os.environ.get("RANK", "0")) == 0:
                print(json.dumps({"impl": "reference", "metric": TRAIN_METRICS[wl["model"]],
                                  "unavailable": "the reference's train step needs myelin@68b8ebb (absent) "
                                                 "for its LIF and spike functions"}), flush=True)
        else:
            run_train(args, wl)
    elif wl.get("kind") == "step":
        if args.impl == "reference":
            run_step_reference(args, wl)
        else:
            run_step(args, wl)
    elif wl.get("kind") == "rwkv7":
        if args.impl == "reference":
            run_rwkv7_reference(args, wl)
        else:
            run_rwkv7(args, wl)
    elif wl.get("kind") == "lif":
        if args.impl == "reference":
            run_lif_reference(args, wl)
        else:
            run_lif(args, wl)
    elif args.incumbent_child:
        run_incumbent_child(args, wl)
    elif args.impl == "reference":
        run_reference(args, wl)
    elif args.sweep_segments:
        run_segment_sweep(args, wl)
    else:
        run_native(args, wl)


if __name__ == "__main__":
    main()
