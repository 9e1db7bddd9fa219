"""Benchmark: bit-exact motion-denoiser steps on B200, through the executor's
C ABI (BASELINE.json metric; configuration 5).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--global-batch G | --batch-per-gpu B]
                    [--impl shlo|reference]

One process per GPU (torchrun for N > 1). By default the global batch G = 512
(the largest of configuration 5's sweep) is split over the ranks (strong
scaling); --batch-per-gpu B gives every rank B samples instead (weak scaling).
Each rank runs the whole 8-layer denoiser module on its share: samples are
independent, so there is no data-path collective. The control plane (barrier,
max over ranks) is torch.distributed over gloo; the one data collective is the
final gather of the results to rank 0 over NCCL, inside the end-to-end loop.

value: sample-steps/s of the whole job with inputs already on the device, timed
with CUDA events on the library's stream, max over ranks. e2e: the same through
the public API with every step's inputs copied from pinned host memory and the
step's whole result brought to rank 0's host memory (gathered over NCCL for
N > 1). roofline: the dominant kernel (mul_mat, ggml_vec_dot_f32 order on FP32
CUDA cores) against the FP32 CUDA-core peak at the SM clock sampled during the
timed region. cpu_baseline / --impl reference: the C oracle (this repo's
restatement of ggml-cpu's arm64 order) on the host cores.
"""
from __future__ import annotations

import argparse
import datetime
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "contract-stablehlo-mlx_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)

import numpy as np  # noqa: E402

METRIC = "bit-exact denoiser steps/s"
UNIT = "sample-steps/s"
WORKLOAD = "8-layer motion denoiser, seq 256, d_model 512, 8 heads, FFN 2048 erf-GELU, timestep MLP (silu)"


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--global-batch", type=int, default=512)
    ap.add_argument("--batch-per-gpu", type=int, default=0, help="weak scaling: this many samples on every GPU")
    ap.add_argument("--layers", type=int, default=8)
    ap.add_argument("--impl", default="shlo", choices=["shlo", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-single-thread", action="store_true", help="skip the single-thread CPU leg")
    # Short runs to wrap in a profiler (no JSON line): one warm denoiser step,
    # mul_mat alone at --mm-shape K,M,R[,N], or every exact kernel once (batch 16).
    ap.add_argument("--profile-run", choices=["step", "mul_mat", "kernels", "attention"])
    ap.add_argument("--mm-shape", default="512,1536,16384")
    return ap.parse_args()


# ----------------------------------------------------------------- clocks ----

class Clocks:
    """nvidia-smi samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu = gpu
        self.rows = []
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), "--query-gpu=" + self.FIELDS,
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unavailable"], "samples": 0}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None
        sm = [num(r[1]) for r in self.rows if num(r[1])]
        mx = [num(r[2]) for r in self.rows if num(r[2])]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows),
                "power_w_max": max([num(r[3]) or 0 for r in self.rows])}


# ------------------------------------------------------------ distributed ----

def dist_init():
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if ws <= 1:
        return 0, 0, 1, None
    import torch.distributed as dist
    dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=300))
    return dist.get_rank(), int(os.environ.get("LOCAL_RANK", "0")), ws, dist


def all_max(dist, v: float) -> float:
    if dist is None:
        return v
    import torch
    t = torch.tensor([v], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(dist):
    if dist is not None:
        dist.barrier()


# -------------------------------------------------------------- peaks ----

def fp32_peak_tflops(device: int) -> float:
    """cuBLAS SGEMM (no TF32) throughput of this GPU, best of several 8192^3."""
    import torch
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    dev = torch.device("cuda", device)
    n = 8192
    a = torch.randn(n, n, device=dev)
    b = torch.randn(n, n, device=dev)
    for _ in range(2):
        torch.matmul(a, b)
    torch.cuda.synchronize(dev)
    best = 0.0
    for _ in range(5):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        torch.matmul(a, b)
        e.record()
        e.synchronize()
        best = max(best, 2 * n ** 3 / (s.elapsed_time(e) * 1e-3) / 1e12)
    del a, b
    torch.cuda.empty_cache()
    return best


def measured_peaks() -> dict:
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return json.load(f)
    except Exception:
        return {}


def profile_traffic(name: str):
    """DRAM bytes per launch of the dominant kernel, and where the figure comes
    from: the ncu capture summarised in profiles/<name> (bench.py cannot run
    ncu itself), with the commit its build was captured at."""
    path = os.path.join(ROOT, "profiles", name)
    val, commit, launch = None, None, None
    try:
        for line in open(path):
            if line.startswith("dram_bytes_per_launch:"):
                val = float(line.split(":", 1)[1].split()[0])
            elif line.startswith("capture_commit:"):
                commit = line.split(":", 1)[1].strip()
            elif line.startswith("capture_launch:"):
                launch = line.split(":", 1)[1].strip()
    except OSError:
        pass
    return val, "ncu capture of %s (profiles/%s), build of commit %s" % (launch or "k_mul_mat_tm", name, commit or "?")


# ------------------------------------------------------------ our arm ----

class EventTimer:
    """CUDA events recorded on the library's own stream."""

    def __init__(self, stream_ptr: int, device: int):
        import torch
        self.torch = torch
        self.stream = torch.cuda.ExternalStream(stream_ptr, device=torch.device("cuda", device))

    def time(self, fn, n: int) -> float:
        t = self.torch
        s, e = t.cuda.Event(enable_timing=True), t.cuda.Event(enable_timing=True)
        s.record(self.stream)
        for _ in range(n):
            fn()
        e.record(self.stream)
        e.synchronize()
        return s.elapsed_time(e) / 1e3  # seconds


def kernel_suite(B: int, cfg, small: bool = False):
    """Every exact kernel at the shape it runs at in this workload (or its BASELINE
    config), as (name, algorithmic bytes, flop, launcher) with the inputs already
    on the device. Bytes: one read of each input + one write of each output."""
    from shlo import mlx as M
    from shlo import run as Run

    rng = np.random.default_rng(7)
    f32 = lambda *s: M.of_numpy((2.0 * rng.standard_normal(s)).astype(np.float32))  # noqa: E731
    out = []
    # [512,1024], N(0, sd 2), 5% -inf, row 0 near 88 (fits in L2)
    x2 = (2.0 * rng.standard_normal((512, 1024))).astype(np.float32)
    x2[rng.random((512, 1024)) < 0.05] = -np.inf
    x2[0] = np.float32(88.0) + rng.uniform(-0.5, 0.5, 1024).astype(np.float32)
    x2[:, 0] = np.where(np.all(np.isinf(x2), axis=1), np.float32(0.0), x2[:, 0])
    a2 = M.of_numpy(x2)
    out.append(("soft_max [512x1024] (config 2)", 2 * 4 * 512 * 1024, 0,
                lambda: Run.soft_max(a2, 1024, 512, 0x3F800000)))
    rows_sm = (B if not small else 16) * cfg.heads * cfg.seq
    asm = f32(rows_sm, cfg.seq)
    out.append(("soft_max [%dx%d] (attention scores)" % (rows_sm, cfg.seq), 2 * 4 * rows_sm * cfg.seq, 0,
                lambda: Run.soft_max(asm, cfg.seq, rows_sm, 0x3F800000)))
    R = (B if not small else 16) * cfg.seq
    an = f32(R, cfg.d)
    out.append(("norm [%dx%d] (layer norm)" % (R, cfg.d), 2 * 4 * R * cfg.d, 0,
                lambda: Run.norm(an, cfg.d, R, 0x3727C5AC)))
    at = f32(B, cfg.d)
    out.append(("silu [%dx%d] (timestep MLP)" % (B, cfg.d), 2 * 4 * B * cfg.d, 0,
                lambda: Run.silu(at, B * cfg.d)))
    ag = f32(R, cfg.ffn)
    out.append(("gelu_erf [%dx%d] (FFN)" % (R, cfg.ffn), 2 * 4 * R * cfg.ffn, 0,
                lambda: Run.gelu_erf(ag, R * cfg.ffn)))
    ne = 1 << (26 if small else 28)
    out.append(("erff_map 2^%d patterns (sweep, config 3)" % (ne.bit_length() - 1), 4 * ne, 0,
                lambda: Run.erff_map(0x3F000000, ne)))
    n32 = 1 << 25
    da, db = f32(n32), f32(n32)
    out.append(("divide 2^25", 3 * 4 * n32, 0, lambda: Run.divide(da, db, n32)))
    out.append(("sqrt 2^25", 2 * 4 * n32, 0, lambda: Run.sqrt(da, n32)))
    n64 = 1 << 24
    fa = M.of_numpy((rng.standard_normal(n64) * 3.0).view(np.uint64), M.dtU64)
    fb = M.of_numpy((rng.standard_normal(n64) * 3.0).view(np.uint64), M.dtU64)
    for op, nm in ((Run.F64_ADD, "add"), (Run.F64_MUL, "mul"), (Run.F64_DIV, "div")):
        out.append(("f64_ew %s 2^24" % nm, 3 * 8 * n64, 0, (lambda o: lambda: Run.f64_ew(o, fa, fb, n64))(op)))
    out.append(("f64_of_f32 2^25", 12 * n32, 0, lambda: Run.f64_of_f32(da, n32)))
    out.append(("f32_of_f64 2^24", 12 * n64, 0, lambda: Run.f32_of_f64(fa, n64)))
    # the fused attention of a layer: q, k, v strided slices of one [B, S, 3, H, 64] projection
    Ba = B if not small else 16
    qkv = f32(Ba, cfg.seq, 3, cfg.heads, cfg.dh)
    qkv_v = [M.reshape(M.slice_(qkv, [0, 0, i, 0, 0], [Ba, cfg.seq, i + 1, cfg.heads, cfg.dh], [1, 1, 1, 1, 1]),
                       [Ba, cfg.seq, cfg.heads, cfg.dh]) for i in range(3)]
    out.append(("attention [%dx%dx%dx%d] (scores, soft_max, value)" % (Ba, cfg.seq, cfg.heads, cfg.dh),
                4 * 4 * Ba * cfg.seq * cfg.heads * cfg.dh, 4 * Ba * cfg.heads * cfg.seq * cfg.seq * cfg.dh,
                lambda: Run.attention(*qkv_v, Ba, cfg.seq, cfg.heads, cfg.dh, cfg.scale_bits())))
    w1, x1 = f32(128, 256), f32(64, 256)
    out.append(("mul_mat [64x256]x[256x128] (config 1)", 4 * (64 * 256 + 256 * 128 + 64 * 128),
                2 * 64 * 128 * 256, lambda: Run.mul_mat(w1, x1, 256, 128, 64, 64, 0)))
    return out


def graph_time(timer, fn, reps: int) -> float:
    """Device seconds per call of `fn`: `reps` calls recorded as one compiled
    function (a CUDA graph) and replayed, so no host work is inside the timing
    (the data stays in L2 between calls where it fits)."""
    from shlo import mlx as M

    def many(args):
        y = None
        for _ in range(reps):
            y = fn()
        return [y]
    fm = M.compile_(many, True)
    M.eval_(M.apply(fm, []))  # records the graph
    M.eval_(M.apply(fm, []))
    t = timer.time(lambda: M.apply(fm, []), 3)
    del fm
    return t / (3 * reps)


def time_kernels(timer, suite, n: int, hbm_gbs: float) -> dict:
    """Per-launch CUDA-event durations on the library's stream, with L2 flushed
    (a 256 MiB fill on the same stream) before every launch; for short kernels
    this includes the host's call overhead. `graph_us`: the device time per
    call, the kernel recorded in a CUDA graph and replayed (graph_time)."""
    torch = timer.torch
    flush = torch.empty(64 << 20, dtype=torch.float32, device=timer.stream.device)
    res = {}
    for name, nbytes, flop, fn in suite:
        for _ in range(2):
            fn()
        total = 0.0
        evs = []
        with torch.cuda.stream(timer.stream):
            for i in range(n):
                flush.fill_(float(i))
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record(timer.stream)
                fn()
                e.record(timer.stream)
                evs.append((s, e))
        timer.stream.synchronize()
        total = sum(s.elapsed_time(e) for s, e in evs) / 1e3
        us = total / n * 1e6
        row = {"us": round(us, 2), "gbs": round(nbytes / (total / n) / 1e9, 1)}
        gt = graph_time(timer, fn, 20 if us < 100 else 5)
        row["graph_us"] = round(gt * 1e6, 2)
        if hbm_gbs:
            row["frac_hbm"] = round(row["gbs"] / hbm_gbs, 3)
        if flop:
            row["tflops"] = round(flop / (total / n) / 1e12, 4)
        res[name] = row
    del flush
    return res


def shard_of(args, ws: int, rank: int):
    """(global batch, this rank's [lo, hi) of it, scaling). Strong scaling by
    default: the global batch is fixed and split over the ranks; with
    --batch-per-gpu every rank takes that many samples (weak scaling)."""
    from shlo import shard as S
    if args.batch_per_gpu:
        G = args.batch_per_gpu * ws
        return G, (rank * args.batch_per_gpu, (rank + 1) * args.batch_per_gpu), "weak"
    G = args.global_batch
    return G, S.split(G, ws, rank), "strong"


class _DeviceView:
    """A library array's storage as a CUDA array for torch (no copy)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3,
                                         "strides": None, "stream": None}


class FinalGather:
    """The one collective of the job: every rank's result rows to rank 0, as
    NCCL sends and receives straight from the library's result storage (no
    kernel reads another GPU's memory), into one global-batch buffer that rank
    0 then copies to pinned host memory. Ordered after the producing step by an
    event on the library's stream; the library's stream is ordered after the
    transfer before the result is released, so its storage is not reused while
    NCCL still reads it."""

    def __init__(self, torch, dist, group, rank, ws, shares, row_elems, lib_stream, device):
        self.torch, self.dist, self.group, self.rank, self.ws = torch, dist, group, rank, ws
        self.counts = [(hi - lo) * row_elems for lo, hi in shares]
        self.offs = [lo * row_elems for lo, _ in shares]
        self.lib_stream = lib_stream
        self.device = device
        self.stream = torch.cuda.Stream(device=device)
        total = sum(self.counts)
        self.big = torch.empty(total, dtype=torch.float32, device=device) if rank == 0 else None
        self.host = torch.empty(total, dtype=torch.float32).pin_memory() if rank == 0 else None
        self.bytes_in = sum(self.counts[1:]) * 4 if rank == 0 else 0

    def __call__(self, M, arr):
        t = self.torch
        ptr, _ = M.device_ptr(arr)
        ready = t.cuda.Event()
        ready.record(self.lib_stream)
        with t.cuda.stream(self.stream):
            self.stream.wait_event(ready)
            mine = t.as_tensor(_DeviceView(ptr, self.counts[self.rank]), device=self.device)
            if self.rank == 0:
                self.big[: self.counts[0]].copy_(mine)
                ops = [self.dist.P2POp(self.dist.irecv, self.big[self.offs[k]: self.offs[k] + self.counts[k]], k,
                                       group=self.group) for k in range(1, self.ws)]
            else:
                ops = [self.dist.P2POp(self.dist.isend, mine, 0, group=self.group)]
            for req in self.dist.batch_isend_irecv(ops):
                req.wait()
            done = t.cuda.Event()
            done.record(self.stream)
            self.lib_stream.wait_event(done)
            if self.rank == 0:
                self.host.copy_(self.big, non_blocking=True)

    def sync(self):
        self.stream.synchronize()


def fp32_nominal_tflops(sm_count: int, sm_mhz: float) -> float:
    """FP32 CUDA-core peak: every SM issues 128 FFMA lanes a cycle (2 flop each)."""
    return sm_count * 128 * 2 * sm_mhz * 1e6 / 1e12


def run_shlo(args):
    rank, local_rank, ws, dist = dist_init()
    import torch

    from shlo import denoiser as D
    from shlo import exec as E
    from shlo import mlx as M  # loads libshlo_cuda (fails loudly without it)
    from shlo import run as Run

    torch.cuda.set_device(local_rank)
    M.set_device(local_rank)
    M.set_flavor("pinned")
    cfg = D.Config(layers=args.layers)
    G, (lo, hi), scaling = shard_of(args, ws, rank)
    B = hi - lo
    shares = [shard_of(args, ws, r)[1] for r in range(ws)]
    w = D.init_weights(cfg, seed=1)
    # The global batch's inputs, seeded once; each rank takes its rows.
    ins_all = D.inputs(cfg, G, seed=1)
    ins = [np.ascontiguousarray(a[lo:hi]) for a in ins_all]
    del ins_all
    W = [M.of_numpy(w[n]) for n, _ in D.weight_specs(cfg)]
    X = [M.of_numpy(a) for a in ins]
    fn = E.prepare(E.load(D.module_text(cfg, B)), None, True)
    timer = EventTimer(M.current_stream(), local_rank)
    nccl = None
    if dist is not None:
        nccl = dist.new_group(backend="nccl", timeout=datetime.timedelta(seconds=300))
        z = torch.zeros(1, device="cuda")
        dist.all_reduce(z, group=nccl)  # the communicator is set up here, outside any timing
        torch.cuda.synchronize()

    def step():
        return M.apply(fn, X + W)[0]

    out = None
    for _ in range(max(args.warmup, 1)):
        out = step()
    M.eval_([out])
    first = M.to_numpy(out)
    out = None

    # ---- value: device-resident inputs, K steps, CUDA events, max over ranks
    holder = []
    barrier(dist)
    torch.cuda.synchronize()
    launches0 = M.launch_count()
    with Clocks(local_rank) as clk:
        dt = timer.time(lambda: holder.__setitem__(slice(None), [step()]), args.steps)
    launches = M.launch_count() - launches0
    last = M.to_numpy(holder[-1])
    holder.clear()
    torch.cuda.synchronize()
    barrier(dist)
    dt_max = all_max(dist, dt)
    deterministic = bool(np.array_equal(first.view(np.uint32), last.view(np.uint32)))

    # ---- e2e: pinned host inputs copied in every step; the step's result read
    # back (N = 1), or gathered to rank 0 over NCCL and read back there (N > 1).
    # Step i's result is read (or gathered) once step i + 1 is queued, so the
    # transfer overlaps the next step's compute; the last one is timed too.
    pinned_in = [torch.from_numpy(a).pin_memory() for a in ins]
    row_elems = cfg.seq * cfg.d
    gather = FinalGather(torch, dist, nccl, rank, ws, shares, row_elems, timer.stream,
                         torch.device("cuda", local_rank)) if ws > 1 else None
    pinned_out = torch.empty(first.shape, dtype=torch.float32).pin_memory() if ws == 1 else None
    out_bytes = B * row_elems * 4

    def finish(o):
        if gather is None:
            M.to_ptr(o, pinned_out.data_ptr(), out_bytes)
        else:
            gather(M, o)

    def e2e_steps(n):
        prev = None
        for _ in range(n):
            xs = [M.of_ptr(p.data_ptr(), p.numel() * 4, list(p.shape), M.dtF32) for p in pinned_in]
            o = M.apply(fn, xs + W)[0]
            if prev is not None:
                finish(prev)
            prev = o
        finish(prev)
        if gather is not None:
            gather.sync()

    e2e_steps(max(args.warmup, 1))
    barrier(dist)
    t0 = time.perf_counter()
    e2e_steps(args.steps)
    e2e_dt = all_max(dist, time.perf_counter() - t0)
    barrier(dist)
    h2d = sum(a.nbytes for a in D.inputs(cfg, 1, seed=1)) * G  # every rank's inputs, whole job
    d2h = G * row_elems * 4                                       # the whole batch's result, read once
    # the gathered batch holds every rank's rows as each rank computed them
    gather_ok = None
    if ws > 1:
        import hashlib
        mine = hashlib.sha256(last.tobytes()).hexdigest()
        digests = [None] * ws
        dist.all_gather_object(digests, mine)
        if rank == 0:
            host = gather.host.numpy()
            gather_ok = all(hashlib.sha256(host[gather.offs[k]: gather.offs[k] + gather.counts[k]].tobytes())
                            .hexdigest() == digests[k] for k in range(ws))

    # ---- batch-1 step latency: the module recorded as a CUDA graph (compile
    # enabled, as the executor prepares it) against plain eager calls
    latency = {}
    X1 = [M.of_numpy(a) for a in D.inputs(cfg, 1, seed=1)]
    for name, comp in (("graph", True), ("eager", False)):
        f1 = E.prepare(E.load(D.module_text(cfg, 1)), None, comp)
        o1 = None
        for _ in range(3):
            o1 = M.apply(f1, X1 + W)[0]
        M.eval_([o1])
        o1 = None
        latency[name] = round(timer.time(lambda: M.apply(f1, X1 + W), 20) / 20 * 1e3, 3)
        del f1
    del X1

    # ---- config 5's batch sweep on one GPU: the step rate at global batches
    # 1, 16 and 64 beside the headline's (compiled, device-resident inputs)
    sweep = {}
    if ws == 1:
        for gb in (1, 16, 64):
            if gb == G:
                continue
            Xb = [M.of_numpy(a) for a in D.inputs(cfg, gb, seed=1)]
            fb = E.prepare(E.load(D.module_text(cfg, gb)), None, True)
            for _ in range(3):
                M.apply(fb, Xb + W)
            nb = 20 if gb <= 16 else 10
            tb = timer.time(lambda: M.apply(fb, Xb + W), nb)
            sweep[str(gb)] = {"sample_steps_per_s": round(gb * nb / tb, 2), "ms_per_step": round(tb / nb * 1e3, 3)}
            del fb, Xb
        sweep[str(G)] = {"sample_steps_per_s": round(G * args.steps / dt, 2), "ms_per_step": round(dt / args.steps * 1e3, 3)}

    # ---- the dominant kernel: mul_mat at a layer's six shapes for this rank's
    # batch (four weight products, then attention's scores and value products,
    # batched per head), each launch with its activation pack
    R = B * cfg.seq
    BH = B * cfg.heads
    rng = np.random.default_rng(0)
    shapes = [(cfg.d, 3 * cfg.d, R, R, 1), (cfg.d, cfg.d, R, R, 1), (cfg.d, cfg.ffn, R, R, 1),
              (cfg.ffn, cfg.d, R, R, 1), (cfg.dh, cfg.seq, BH * cfg.seq, cfg.seq, BH),
              (cfg.seq, cfg.dh, BH * cfg.seq, cfg.seq, BH)]
    mm_flops, mm_time, mm_launches = 0.0, 0.0, 0
    per_shape = {}
    weight_flops, weight_time = 0.0, 0.0
    for K, Mm, Rr, Nn, Wb in shapes:
        wa = M.of_numpy(rng.standard_normal((Wb * Mm, K)).astype(np.float32))
        xa = M.of_numpy(rng.standard_normal((Rr, K)).astype(np.float32))
        wbs = Mm * K if Wb > 1 else 0
        for _ in range(3):
            y = Run.mul_mat(wa, xa, K, Mm, Rr, Nn, wbs)
        M.eval_([y])
        n = 10
        t = timer.time(lambda: Run.mul_mat(wa, xa, K, Mm, Rr, Nn, wbs), n)
        mm_flops += 2.0 * K * Mm * Rr * n
        mm_time += t
        mm_launches += n
        if Wb == 1:
            weight_flops += 2.0 * K * Mm * Rr * n
            weight_time += t
        per_shape["%s%dx%dx%d" % ("%dx" % Wb if Wb > 1 else "", Rr // Wb, Mm, K)] = round(
            2.0 * K * Mm * Rr / (t / n) / 1e12, 2)
        del wa, xa, y
    mm_tflops = mm_flops / mm_time / 1e12
    weight_tflops = weight_flops / weight_time / 1e12
    # Small products, timed on the device: n calls recorded as one CUDA graph
    # (a compiled function) and replayed, so the host's per-call overhead is
    # not in the figure. Config 1, the timestep MLP's products at this rank's
    # batch, and a layer's products at batch 1 (the latency case).
    small = {}
    for name, (K, Mm, Rr) in (("config1 64x256x128", (256, 128, 64)),
                              ("timestep %dx512x512" % B, (cfg.d, cfg.d, B)),
                              ("batch1 qkv 256x1536x512", (cfg.d, 3 * cfg.d, cfg.seq)),
                              ("batch1 ffn2 256x512x2048", (cfg.ffn, cfg.d, cfg.seq))):
        wa = M.of_numpy(rng.standard_normal((Mm, K)).astype(np.float32))
        xa = M.of_numpy(rng.standard_normal((Rr, K)).astype(np.float32))
        reps = 50

        def many(args, K=K, Mm=Mm, Rr=Rr):
            y = None
            for _ in range(reps):
                y = Run.mul_mat(args[0], args[1], K, Mm, Rr, Rr, 0)
            return [y]
        fm = M.compile_(many, True)
        M.eval_(M.apply(fm, [wa, xa]))  # records the graph
        t = timer.time(lambda: M.apply(fm, [wa, xa]), 5)
        small[name] = {"us_per_call": round(t / (5 * reps) * 1e6, 2),
                       "tflops": round(2.0 * K * Mm * Rr * 5 * reps / t / 1e12, 3)}
        del fm, wa, xa
    # dot_general config 1: [64,256] x [256,128]
    w1 = M.of_numpy(rng.standard_normal((128, 256)).astype(np.float32))
    x1 = M.of_numpy(rng.standard_normal((64, 256)).astype(np.float32))
    for _ in range(5):
        Run.mul_mat(w1, x1, 256, 128, 64, 64, 0)
    n1 = 200
    t1 = timer.time(lambda: Run.mul_mat(w1, x1, 256, 128, 64, 64, 0), n1)
    cfg1_tflops = 2.0 * 64 * 128 * 256 / (t1 / n1) / 1e12

    kernels = time_kernels(timer, kernel_suite(64, cfg), 10, measured_peaks().get("hbm_gbs"))

    sgemm = fp32_peak_tflops(local_rank)
    sm_count = torch.cuda.get_device_properties(local_rank).multi_processor_count
    clocks = clk.summary()
    sm_mhz = clocks.get("sm_mhz") or clocks.get("sm_max_mhz") or measured_peaks().get("sm_max_mhz") or 1965.0
    peak = fp32_nominal_tflops(sm_count, sm_mhz)
    peak_max = fp32_nominal_tflops(sm_count, clocks.get("sm_max_mhz") or measured_peaks().get("sm_max_mhz") or 1965.0)

    if rank != 0:
        if dist is not None:
            dist.barrier()
            dist.destroy_process_group()
        return

    # ---- CPU baselines (rank 0, N = 1): the oracle on one sample through every
    # layer, rows split over all host cores, and on one thread (ggml_ref's mode)
    cpu = cpu1 = None
    exact0 = None
    if ws == 1 and not args.no_cpu_baseline:
        from oracle import model_oracle as MO
        cores = os.cpu_count() or 1
        one = [a[:1] for a in ins]
        t = time.perf_counter()
        ref0 = MO.forward(cfg, w, one, nthreads=cores)
        cdt = time.perf_counter() - t
        exact0 = bool(np.array_equal(ref0.view(np.uint32), first[:1].view(np.uint32)))
        cpu = {"value": round(1.0 / cdt, 4), "unit": UNIT, "cores": cores, "kind": "port",
               "sample": "one sample (batch 1) through all %d layers on the C oracle, rows split over %d host threads; "
                         "%.1f s" % (cfg.layers, cores, cdt)}
        if not args.no_single_thread:
            t = time.perf_counter()
            MO.forward(cfg, w, one, nthreads=1)
            cdt1 = time.perf_counter() - t
            cpu1 = {"value": round(1.0 / cdt1, 4), "unit": UNIT, "cores": 1, "kind": "port",
                    "sample": "one sample through all %d layers on the C oracle on one thread (ggml_ref's own "
                              "single-thread mode); %.1f s" % (cfg.layers, cdt1)}

    value = G * args.steps / dt_max
    flops_step = cfg.flops_per_sample() * G
    traffic, traffic_note = profile_traffic("mul_mat_denoiser_qkv.md")
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": ws, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": round(dt_max / args.steps * 1e3, 3), "higher_is_better": True,
        "scaling": scaling, "vs_baseline": None, "dtype": "f32",
        "data": "synthetic: seeded N(0,1) noisy inputs and host sinusoid timestep embeddings, N(0,0.02) random-init weights",
        "config": config_of(cfg, G, ws, scaling),
        "batch_per_gpu": B,
        "model_tflops": round(flops_step * args.steps / dt_max / 1e12, 2),
        "roofline": {"bound": "fp32-cuda-core",
                     "kernel": "mul_mat (k_mm_pack of x + k_mul_mat_tm) at the step's four weight products of a layer "
                               "(QKV, output, FFN1, FFN2; attention's products run inside k_attention)",
                     "achieved": round(weight_tflops, 2), "peak": round(peak, 2), "unit": "TFLOP/s",
                     "frac": round(weight_tflops / peak, 3),
                     "peak_source": "FP32 CUDA-core peak: %d SMs x 128 FFMA lanes x 2 flop x %.0f MHz (median SM clock "
                                    "sampled during the timed region; MEASURED_PEAKS.json has no FP32 figure)"
                                    % (sm_count, sm_mhz),
                     "peak_at_max_clock": round(peak_max, 2), "frac_at_max_clock": round(weight_tflops / peak_max, 3),
                     "six_shapes_tflops": round(mm_tflops, 2),
                     "six_shapes_note": "the four weight products and, as standalone mul_mat calls, attention's scores "
                                        "and value shapes (the unfused path's)",
                     "sgemm_tflops": round(sgemm, 2),
                     "sgemm_note": "cuBLAS SGEMM (TF32 off) 8192^3 on this GPU in this run, a side note: not the peak",
                     "per_shape": per_shape,
                     "traffic": traffic, "traffic_source": traffic_note},
        "kernels": kernels,
        "dot_general": {"config1_64x256x128_tflops": round(cfg1_tflops, 4),
                        "config1_us_per_call": round(t1 / n1 * 1e6, 2),
                        "config1_note": "eager calls from Python through the C ABI, host overhead included; "
                                        "small_products has the device time",
                        "denoiser_shapes_tflops": round(mm_tflops, 2),
                        "small_products": small},
        "cpu_baseline": cpu,
        "cpu_baseline_single_thread": cpu1,
        "e2e": {"value": round(G * args.steps / e2e_dt, 3), "unit": UNIT, "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "final_gather": None if ws == 1 else {"how": "NCCL send/recv of every rank's result rows to rank 0, "
                                                             "then one device-to-host copy of the global batch",
                                                      "nvlink_bytes_per_step": gather.bytes_in,
                                                      "gathered_equals_ranks_results": gather_ok}},
        "gpu_launches": int(launches),
        "latency_b1_ms": latency,
        "batch_sweep_1gpu": sweep or None,
        "clocks": clocks,
        "bit_exact": {"sample0_vs_oracle": exact0, "deterministic_across_steps": deterministic},
        "hbm_gbs_measured": measured_peaks().get("hbm_gbs"),
    }
    print(json.dumps(line), flush=True)
    if dist is not None:
        dist.barrier()
        dist.destroy_process_group()


def config_of(cfg, G, ws, scaling):
    return {"workload": WORKLOAD, "global_batch": G, "seq_len": cfg.seq, "layers": cfg.layers,
            "parallelism": "dp%d (%s scaling: independent batch shards, no collective but the final gather)"
                           % (ws, scaling),
            "l2": "no flush: per-step working set (100 MB weights + >1 GB activations) exceeds the 126 MB L2",
            "ggml_build": "pinned"}


# ------------------------------------------------------ the reference arm ----

def run_reference(args):
    """The reference's CPU path for this workload: the C oracle (ggml-cpu's arm64
    order restated; the reference's own ggml_ref cannot be built here), one
    sample of the same global batch per step through all layers, rows split
    over every host thread. Rank 0 alone runs; the other ranks exit at once.
    Nothing here maps the CUDA library: `shlo.denoiser` and `shlo.shard` are
    host-only modules."""
    rank = int(os.environ.get("RANK", "0"))
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from oracle import model_oracle as MO
    from shlo import denoiser as D

    cfg = D.Config(layers=args.layers)
    G, _, scaling = shard_of(args, ws, 0)
    w = D.init_weights(cfg, seed=1)
    ins = [a[:1] for a in D.inputs(cfg, 1, seed=1)]
    cores = os.cpu_count() or 1
    for _ in range(args.warmup):
        MO.forward(cfg, w, ins, nthreads=cores)
    t = time.perf_counter()
    for _ in range(args.steps):
        MO.forward(cfg, w, ins, nthreads=cores)
    dt = time.perf_counter() - t
    v = args.steps / dt
    line = {"metric": METRIC, "value": round(v, 4), "unit": UNIT, "impl": "reference", "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 1),
            "higher_is_better": True, "scaling": scaling, "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded N(0,1) noisy inputs and host sinusoid timestep embeddings, N(0,0.02) random-init weights",
            "config": config_of(cfg, G, ws, scaling),
            "cpu_baseline": {"value": round(v, 4), "unit": UNIT, "cores": cores, "kind": "port",
                             "sample": "each step: one sample of the batch through all %d layers on the C oracle, "
                                       "rows split over %d host threads (the rate is per sample)" % (cfg.layers, cores)},
            "e2e": {"value": round(v, 4), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def profile_run(args):
    """A short, fixed piece of work for `ncu` to capture (see profiles/)."""
    import shlo  # noqa: F401
    from shlo import denoiser as D
    from shlo import exec as E
    from shlo import mlx as M
    from shlo import run as Run

    M.set_flavor("pinned")
    if args.profile_run == "step":
        cfg = D.Config(layers=args.layers)
        B = args.batch_per_gpu or 64
        w = D.init_weights(cfg, seed=1)
        W = [M.of_numpy(w[n]) for n, _ in D.weight_specs(cfg)]
        X = [M.of_numpy(a) for a in D.inputs(cfg, B, seed=1)]
        # compiled, as the executor prepares it: the first call runs the trace
        # eagerly and records the fused graph, the second replays it (the graph's
        # kernels are the last launches of the run)
        fn = E.prepare(E.load(D.module_text(cfg, B)), None, True)
        c0 = M.launch_count()
        M.eval_([M.apply(fn, X + W)[0]])  # warm-up step (eager trace + recording)
        c1 = M.launch_count()
        M.eval_([M.apply(fn, X + W)[0]])  # the replayed step
        print("launches: warm-up %d, step %d" % (c1 - c0, M.launch_count() - c1))
    elif args.profile_run == "attention":
        # the fused attention at batch 16 of the denoiser's shape, three launches
        cfg = D.Config(layers=1)
        B = 16
        rng = np.random.default_rng(0)
        qkv = M.of_numpy(rng.standard_normal((B, cfg.seq, 3, cfg.heads, cfg.dh)).astype(np.float32))
        qkv_v = [M.reshape(M.slice_(qkv, [0, 0, i, 0, 0], [B, cfg.seq, i + 1, cfg.heads, cfg.dh], [1, 1, 1, 1, 1]),
                           [B, cfg.seq, cfg.heads, cfg.dh]) for i in range(3)]
        outs = [Run.attention(*qkv_v, B, cfg.seq, cfg.heads, cfg.dh, cfg.scale_bits()) for _ in range(3)]
        M.eval_(outs)
        print("attention [%dx%dx%dx%d]: 3 launches" % (B, cfg.seq, cfg.heads, cfg.dh))
    elif args.profile_run == "kernels":
        suite = kernel_suite(args.batch_per_gpu or 64, D.Config(layers=args.layers), small=True)
        outs = [fn() for _, _, _, fn in suite]
        M.eval_(outs)
        print("kernels: %d launches: %s" % (len(suite), "; ".join(n for n, _, _, _ in suite)))
    else:
        # K,M,R (one shared w) or K,M,R,N (R / N batches, each with its own w)
        dims = [int(v) for v in args.mm_shape.split(",")]
        K, Mm, R = dims[:3]
        N = dims[3] if len(dims) > 3 else R
        nb = R // N if len(dims) > 3 else 1
        rng = np.random.default_rng(0)
        wa = M.of_numpy(rng.standard_normal((nb * Mm, K)).astype(np.float32))
        xa = M.of_numpy(rng.standard_normal((R, K)).astype(np.float32))
        wbs = Mm * K if nb > 1 else 0
        for _ in range(3):
            y = Run.mul_mat(wa, xa, K, Mm, R, N, wbs)
        M.eval_([y])
        print("mul_mat %s: 3 launches" % args.mm_shape)


def main():
    args = parse_args()
    if args.profile_run:
        profile_run(args)
        return
    if args.impl == "reference":
        run_reference(args)
    else:
        run_shlo(args)


if __name__ == "__main__":
    main()
