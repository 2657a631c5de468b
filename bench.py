"""Benchmark: atom-evaluations per second (energy + forces) of the SOG mesh solver.

Workload (default, the large single system): 1,048,576 atoms uniform in a
cubic 220 A cell, neutral N(0, 0.6) charges, 12 Gaussians with bandwidths
log-spaced 1.2-60 A and raw amplitudes 1/(bw sqrt(2 pi)), n_dl = 0.86 -> 512^3
mesh, cardinal B-spline order 6, float64.  Synthetic, seeded (seed 0 + rank).

One step = one energy + explicit-force evaluation of the whole system.
  value   device throughput, inputs resident in HBM (CUDA events, max over ranks)
  e2e     the same through the public API (sog_b200.Sog) with pinned host
          inputs copied in and energy + forces copied out every step
With N > 1 ranks (torchrun) the system's mesh is split into z slabs over the
GPUs (--mode slab, default: strong scaling), or every rank solves its own
independent system (--mode frames: weak scaling).

--config cfg4 times the batched-frames workload instead: 512 independent
cubic frames of 200-5000 atoms (density 0.1 / A^3, n_dl = 1.0, per-frame
meshes 25^3-75^3, B-spline order 6); with N ranks the frames are shared out
by the longest-processing-time rule (sog_b200.shard), no collective on the
data path: strong scaling of the fixed batch.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl sog_b200|reference]
                    [--config cfg5|cfg5_eighth|cfg5_quarter|cfg2|cfg4] [--dtype f64|f32] [--eager]
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "atom-evals/sec (E+F)"
UNIT = "atom-evals/s"


# ---------------------------------------------------------------------------
# workload
# ---------------------------------------------------------------------------
def workload(name: str):
    if name == "cfg5":
        return dict(workload="large single system: 1,048,576 atoms, 220 A cubic, 512^3 mesh, "
                             "B-spline order 6, 12 Gaussians bw 1.2-60 A", natoms=1 << 20, L=220.0,
                    n_dl=0.86, order=6, m=12, bw_lo=1.2, bw_hi=60.0, qstd=0.6)
    if name == "cfg5_eighth":
        return dict(workload="1/8-scale large system: 131,072 atoms, 110 A cubic, 256^3 mesh, "
                             "B-spline order 6, 12 Gaussians bw 1.2-60 A", natoms=1 << 17, L=110.0,
                    n_dl=0.86, order=6, m=12, bw_lo=1.2, bw_hi=60.0, qstd=0.6)
    if name == "cfg5_quarter":
        return dict(workload="quarter-height slab of the large system: 262,144 atoms, 220 x 220 x 55 A, "
                             "512 x 512 x 128 mesh, B-spline order 6, 12 Gaussians bw 1.2-60 A "
                             "(profiling case: about 3 GB on the device)", natoms=1 << 18, L=220.0,
                    box=(220.0, 220.0, 55.0), n_dl=0.86, order=6, m=12, bw_lo=1.2, bw_hi=60.0, qstd=0.6)
    if name == "cfg5_zslab":
        return dict(workload="half-width column of the large system: 262,144 atoms, 110 x 110 x 220 A, "
                             "256 x 256 x 512 mesh, B-spline order 6, 12 Gaussians bw 1.2-60 A "
                             "(profiling case for the 512-point z pass: about 3 GB on the device)",
                    natoms=1 << 18, L=220.0, box=(110.0, 110.0, 220.0), n_dl=0.86, order=6, m=12,
                    bw_lo=1.2, bw_hi=60.0, qstd=0.6)
    if name == "cfg2":
        return dict(workload="water-like box: 3,000 atoms, 31 A cubic, 64^3 mesh, B-spline order 6, "
                             "12 Gaussians bw 1.2*1.62^m", natoms=3000, L=31.0, n_dl=1.0, order=6,
                    m=12, bw_geom=(1.2, 1.62), qstd=None)
    raise SystemExit(f"unknown config {name}")


def make_batch(seed: int = 0, nframes: int = 512):
    """Batched-frames workload: frame sizes U{200..5000}, cubic cells of
    density 0.1 atoms / A^3, uniform positions, U(-1, 1) charges neutral per
    frame, 12 Gaussians bw 1.2 * 1.62^m with raw amplitudes."""
    import numpy as np
    rng = np.random.default_rng(seed)
    ns = rng.integers(200, 5001, nframes)
    rs, qs, cells = [], [], []
    for n in ns:
        L = (n / 0.1) ** (1.0 / 3.0)
        rs.append(rng.random((n, 3)) * L)
        qq = rng.uniform(-1.0, 1.0, n)
        qs.append(qq - qq.mean())
        cells.append(np.eye(3) * L)
    bw = 1.2 * 1.62 ** np.arange(12)
    amp_raw = 1.0 / (bw * math.sqrt(2.0 * math.pi))
    return [int(n) for n in ns], np.concatenate(rs), np.concatenate(qs), np.stack(cells), amp_raw, bw


def bucket_bytes(dims, nframes: int, natoms: int, s: int = 8, nfield: int = 3):
    """Minimal-pipeline bytes per kernel name of one mesh bucket (the same
    accounting as algorithmic_bytes, for nframes frames of one mesh)."""
    nx, ny, nz = dims
    ng = nx * ny * nz * nframes
    nh = nz * ny * (nx // 2 + 1) * nframes
    N = natoms
    out = {
        "spread": s * ng + 4 * s * N,
        "fft_r2c_x": s * ng + 2 * s * nh,
        "fft_y_fwd": 4 * s * nh,
        "fft_y_inv": (2 + nfield) * 2 * s * nh if nz & (nz - 1) == 0 else nfield * 4 * s * nh,
        "fft_c2r_x": nfield * (2 * s * nh + s * ng),
        "gather": nfield * s * ng + 7 * s * N,
        "green": s * nh,
    }
    if nz & (nz - 1) == 0:        # fused z pass: spectrum in, Y1 and Y2 out
        out["zfused"] = 2 * s * nh + 2 * 2 * s * nh
    else:                         # z passes around the k-space kernel
        out.update({"fft_z_fwd": 4 * s * nh, "kspace": 2 * s * nh + nfield * 2 * s * nh,
                    "fft_z_inv": nfield * 4 * s * nh})
    return out, 7 * s * N + 8 * s * ng + 16 * s * nh


def make_inputs(cfg, seed: int):
    import numpy as np
    rng = np.random.default_rng(seed)
    n, L = cfg["natoms"], cfg["L"]
    box = np.array(cfg.get("box", (L, L, L)))
    r = rng.random((n, 3)) * box
    if cfg.get("qstd"):
        q = rng.standard_normal(n) * cfg["qstd"]
    else:
        q = np.where(np.arange(n) % 3 == 0, -0.8, 0.4) + 0.05 * rng.standard_normal(n)
    q -= q.mean()
    if "bw_geom" in cfg:
        b0, f = cfg["bw_geom"]
        bw = b0 * f ** np.arange(cfg["m"])
    else:
        bw = np.logspace(math.log10(cfg["bw_lo"]), math.log10(cfg["bw_hi"]), cfg["m"])
    amp_raw = 1.0 / (bw * math.sqrt(2.0 * math.pi))
    cell = np.diag(box)
    return r, q, cell, amp_raw, bw


def mesh_dims(cfg):
    """(nx, ny, nz) of the n_dl grid rule for the workload's box."""
    dims = []
    for L in cfg.get("box", (cfg["L"],) * 3):
        n = 2 * int(math.floor(L / cfg["n_dl"])) + 1
        while True:
            m = n
            for p in (2, 3, 5):
                while m % p == 0:
                    m //= p
            if m == 1:
                break
            n += 1
        dims.append(n)
    return tuple(dims)


def algorithmic_bytes(cfg, s: int = 8, nfield: int = 3, parts: int = 1):
    """Minimal-pipeline bytes per evaluation (each array once per producer /
    consumer pass) and per kernel launch; with the mesh split into `parts`
    slabs, the per-launch figures of one rank."""
    nx, ny, nz = mesh_dims(cfg)
    N = cfg["natoms"]
    ng = nx * ny * nz
    nh = nz * ny * (nx // 2 + 1)
    per_kernel = {
        "spread": s * ng + 4 * s * N,
        "fft_r2c_x": s * ng + 2 * s * nh,
        "fft_y_fwd": 4 * s * nh,
        "fft_z_fwd": 4 * s * nh,
        "kspace": 2 * s * nh + nfield * 2 * s * nh,
        "fft_z_inv": nfield * 4 * s * nh,
        # inverse y pass of an orthorhombic frame with forces: the two z-pass
        # outputs Y1, Y2 in, the three ik fields out
        "fft_y_inv": (2 + nfield) * 2 * s * nh,
        "fft_c2r_x": nfield * (2 * s * nh + s * ng),
        "gather": nfield * s * ng + 4 * s * N + 3 * s * N,
        # fused z pass: spectrum in, the two field spectra Y1, Y2 out (the
        # Green function comes from a radial table in L2: no HBM bytes)
        "zfused": 2 * s * nh + 2 * 2 * s * nh,
        # Green table written once per evaluation
        "green": s * nh,
    }
    b_ef = 7 * s * N + 8 * s * ng + 16 * s * nh
    if parts > 1:
        per_kernel = {k: v / parts for k, v in per_kernel.items()}
        b_ef = b_ef / parts
    return b_ef, per_kernel


def profiled_traffic(kernel: str, config: str):
    """DRAM bytes per launch of `kernel` at 512^3 from the committed ncu
    summary (profiles/dram_mesh256x256x512_bspline6.md: captured on the
    quarter-size profiling case, scaled by the algorithmic-bytes ratio), or
    None.  A figure copied from that capture, not a measurement of the
    current run; the JSON line says so next to it."""
    if config != "cfg5":
        return None
    p = os.path.join(ROOT, "profiles", TRAFFIC_PROFILE)
    try:
        with open(p) as f:
            for line in f:
                cells = [c.strip().strip("`") for c in line.strip().strip("|").split("|")]
                if len(cells) >= 10 and cells[1] == kernel:
                    return float(cells[9]) * 1e9
    except (OSError, ValueError):
        return None
    return None


TRAFFIC_PROFILE = "dram_mesh256x256x512_bspline6.md"


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def measured_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


# ---------------------------------------------------------------------------
# clocks sampling during the timed region
# ---------------------------------------------------------------------------
class ClockSampler:
    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []
        self.t = None

    def start(self):
        # nvidia-smi writes to a file: no reader thread competes with the
        # launching thread during the timed region
        import tempfile
        self.path = tempfile.mktemp(prefix="sog_clocks_", suffix=".csv")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                 "--format=csv,noheader,nounits", "-lms", "200", "-f", self.path],
                stdout=subprocess.DEVNULL, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        # nvidia-smi's start-up (driver and NVML initialisation) can hold the
        # driver for a while; wait for its first sample so that it is not
        # under way inside the timed region
        t0 = time.time()
        while time.time() - t0 < 10.0:
            try:
                if os.path.getsize(self.path) > 0:
                    break
            except OSError:
                pass
            time.sleep(0.05)

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        try:
            with open(self.path) as fh:
                self.lines = [ln.strip() for ln in fh if ln.strip()]
            os.remove(self.path)
        except Exception:
            self.lines = []
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


# ---------------------------------------------------------------------------
# CPU oracle timing (cpu_baseline and the reference arm)
# ---------------------------------------------------------------------------
def oracle_eval_time(cfg_name: str, reps: int, warm: int = 1):
    """E+F of the workload `cfg_name` by the C/OpenMP oracle on every host
    core; returns (cfg, per-evaluation seconds, threads, last result with the
    k=0 term added to its energy)."""
    import numpy as np
    from oracle import oracle as O
    threads = O.set_num_threads(host_cores())
    cfg = workload(cfg_name)
    r, q, cell, amp_raw, bw = make_inputs(cfg, 0)
    nx, ny, nz = mesh_dims(cfg)
    amp = amp_raw * bw * bw
    ksm = (2.0 * math.pi / cfg["n_dl"]) ** 2
    times = []
    res = None
    for i in range(warm + reps):
        t0 = time.perf_counter()
        res = O.mesh_solve(r, q, cell, amp, bw * bw, spline=O.BSPLINE, order=cfg["order"], nx=nx,
                           ny=ny, nz=nz, k_sq_max=ksm, want_force=True)
        dt = time.perf_counter() - t0
        if i >= warm:
            times.append(dt)
    e0, _, _, _ = O.k0_correction(q[:, None], cell, amp, bw * bw, norm_factor=14.3996454784255,
                                  remove_self=True)
    res["energy"] += e0
    return cfg, times, threads, res


def reference_torch_time(cfg_name: str, reps: int = 2, warm: int = 1):
    """The reference's own torch CPU path on the same sample: QuadS order 6
    with explicit E+F through Gaussian.compute_bundle (batched direct gate
    off), fp64, torch threads = host cores.  Runs the reference installed in
    baseline/_ref; None when it is not there."""
    path = os.path.join(ROOT, "baseline", "_ref")
    if not os.path.isdir(os.path.join(path, "sog")):
        return None
    import warnings
    import torch
    if path not in sys.path:
        sys.path.insert(0, path)
    with warnings.catch_warnings():
        warnings.simplefilter("ignore")
        from sog.module.gaussian import Gaussian as RefGaussian
        cores = host_cores()
        torch.set_num_threads(cores)
        cfg = workload(cfg_name)
        r, q, cell, amp_raw, bw = make_inputs(cfg, 0)
        g = RefGaussian(n_dl=cfg["n_dl"], amp=torch.tensor(amp_raw), bandwidth=torch.tensor(bw),
                        use_quads_fft=True, quads_order=cfg["order"], trainable=False)
        g._enable_batched_direct = False
        rt, qt = torch.tensor(r), torch.tensor(q)
        ct = torch.tensor(cell).unsqueeze(0)
        bt = torch.zeros(len(r), dtype=torch.long)
        times = []
        for i in range(warm + reps):
            t0 = time.perf_counter()
            with torch.no_grad():
                g.compute_bundle(q=qt, r=rt, cell=ct, batch=bt, compute_force=True)
            if i >= warm:
                times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": cfg["natoms"] / t, "unit": UNIT, "cores": cores, "kind": "reference",
            "sample": f"{cfg['workload']}; the reference's torch QuadS-{cfg['order']} explicit E+F "
                      f"(compute_bundle, batched direct gate off), median of {reps} after {warm} "
                      f"warm-up, {t:.2f} s per evaluation",
            "note": "QuadS: the reference's Python solvers have no B-spline mesh"}


def oracle_batch_time(frames: int = 120):
    """The oracle's E+F on the first `frames` frames of the batched workload."""
    from oracle import oracle as O
    from tests._cases import friendly
    O.set_num_threads(host_cores())
    counts, r, q, cells, amp_raw, bw = make_batch(0)
    amp = amp_raw * bw * bw
    ksm = (2.0 * math.pi / 1.0) ** 2
    t, atoms, b = 0.0, 0, 0
    for j in range(frames):
        n = counts[j]
        L = float(cells[j][0, 0])
        g = friendly(max(8, 2 * int(math.floor(L / 1.0)) + 1))
        t0 = time.perf_counter()
        O.mesh_solve(r[b:b + n], q[b:b + n], cells[j], amp, bw * bw, spline=O.BSPLINE, order=6,
                     nx=g, ny=g, nz=g, k_sq_max=ksm, want_force=True)
        t += time.perf_counter() - t0
        atoms += n
        b += n
    return atoms, t, O.num_threads()


def run_reference(args, rank: int):
    if rank != 0:
        return
    if args.config == "cfg4":
        atoms, t, threads = oracle_batch_time()
        val = atoms / t
        line = {
            "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus, "steps": 1,
            "warmup": 0, "ms_per_step": t * 1e3, "higher_is_better": True, "scaling": "strong",
            "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded)", "impl": "reference",
            "config": {"workload": BATCH_WORKLOAD, "sample": f"first 120 frames ({atoms} atoms)"},
            "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                             "sample": f"first 120 frames of the batch ({atoms} atoms), E+F by the "
                                       "C/OpenMP oracle"},
            "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line), flush=True)
        return
    sample = "cfg5_eighth"
    cfg, times, threads, _ = oracle_eval_time(sample, reps=args.steps, warm=args.warmup)
    t = statistics.median(times)
    val = cfg["natoms"] / t
    main_cfg = workload(args.config)
    line = {
        "metric": METRIC, "value": val, "unit": UNIT, "n_gpus": args.gpus, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": t * 1e3, "higher_is_better": True,
        "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic (seeded)",
        "impl": "reference",
        "config": {"workload": main_cfg["workload"], "sample": cfg["workload"]},
        "cpu_baseline": {"value": val, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{cfg['workload']}; one E+F evaluation per step by the C/OpenMP "
                                   "oracle (the reference's B-spline mesh restated), median of steps"},
        "e2e": {"value": val, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "reference_torch": reference_torch_time(sample),
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU arm
# ---------------------------------------------------------------------------
BATCH_WORKLOAD = ("batched frames: 512 cubic frames of 200-5000 atoms (1,382,639 atoms), density "
                  "0.1/A^3, n_dl 1.0 (meshes 25^3-75^3), B-spline order 6, 12 Gaussians "
                  "bw 1.2*1.62^m")


def run_gpu_batch(args, rank: int, world: int):
    """Batched independent frames, shared out over the ranks by LPT."""
    import numpy as np
    import torch
    import torch.distributed as dist

    from sog_b200 import Sog, _lib
    from sog_b200.grid import resolve_grid
    from sog_b200.shard import FrameShards, frame_costs, lpt_partition

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dt = torch.float64 if args.dtype == "f64" else torch.float32
    s = 8 if dt == torch.float64 else 4
    counts, r, q, cells, amp_raw, bw = make_batch(0)
    import warnings
    with warnings.catch_warnings():
        warnings.simplefilter("ignore", DeprecationWarning)
        grids = [resolve_grid(*(float(c[i, i]) for i in range(3)), n_dl=1.0, cubes2_phi_max=None,
                              r_c=None, min_grid=8)[:3] for c in cells]
    costs = frame_costs(counts, [g[0] * g[1] * g[2] for g in grids], order=6)
    sh = FrameShards(counts, lpt_partition(costs, world), rank, dev)
    model = Sog({"use_atomwise": False, "use_bspline_fft": True, "bspline_order": 6, "n_dl": 1.0,
                 "amp": torch.tensor(amp_raw, dtype=dt), "bandwidth": torch.tensor(bw, dtype=dt),
                 "trainable_kernel": False}).to(dev)
    gauss = model.gaussian
    r_all = torch.tensor(r, dtype=dt, device=dev)
    q_all = torch.tensor(q, dtype=dt, device=dev)[:, None]
    c_all = torch.tensor(cells, dtype=dt, device=dev)
    r_d, q_d, c_d, b_d = sh.select(r_all, q_all, c_all)
    del r_all, q_all
    N = int(r_d.shape[0])
    nf_local = len(sh.frames)

    def barrier():
        if world > 1:
            dist.barrier()

    def align_streams():
        # after the host barrier the ranks leave at slightly different times;
        # a one-element sum enqueued right before the first event lines up
        # the GPUs' streams themselves, so the first timed step does not
        # absorb the host-side release skew
        if world > 1:
            dist.all_reduce(torch.zeros(1, device=dev))

    def step_device():
        return gauss.compute_bundle(q=q_d, r=r_d, cell=c_d, batch=b_d, compute_force=True)

    for _ in range(max(1, args.warmup)):
        step_device()
    torch.cuda.synchronize()
    lay = gauss._layout
    plans = [p for p in _lib.PLANS.plans.values()
             if any(p.key[4] == tuple(b.dims) for b in lay["buckets"])]
    for p in plans:
        p.set_timing(True)
    stream = torch.cuda.current_stream()
    # every rank starts its clock sampler first; the barrier right before the
    # first event then lines the ranks up, so no rank's sampler start-up
    # lands inside another rank's first timed step
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    gc.collect()
    gc.disable()
    barrier()
    torch.cuda.synchronize()
    align_streams()
    l0 = _lib.launch_count()
    ev0.record(stream)
    h0 = time.perf_counter()
    for _ in range(args.steps):
        out = step_device()
    host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
    ev1.record(stream)
    torch.cuda.synchronize()
    gc.enable()
    launches = _lib.launch_count() - l0
    clk = clocks.stop()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    tot, cnt = {}, {}
    for p in plans:
        for name, t in p.timings():
            tot[name] = tot.get(name, 0.0) + t
            cnt[name] = cnt.get(name, 0) + 1
        p.set_timing(False)
    ms_all = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_all, op=dist.ReduceOp.MAX)
    ms_max = float(ms_all.item())
    e_sum = float(out["energy"].sum())

    # ---- end to end through Sog.forward with this rank's share in pinned host memory ----
    r_h = r_d.cpu().pin_memory()
    q_h = q_d[:, 0].cpu().pin_memory()
    e_h = torch.empty(nf_local, dtype=dt).pin_memory()
    f_h = torch.empty(N, 3, dtype=dt).pin_memory()
    r_in = torch.empty_like(r_d)
    q_in = torch.empty(N, dtype=dt, device=dev)

    def step_e2e():
        r_in.copy_(r_h, non_blocking=True)
        q_in.copy_(q_h, non_blocking=True)
        o = model(positions=r_in, cell=c_d, latent_charges=q_in, batch=b_d, compute_force=True)
        e_h.copy_(o["E_lr"], non_blocking=True)
        f_h.copy_(o["forces"], non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step_e2e()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step_e2e()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_e2e, op=dist.ReduceOp.MAX)
    ms_e2e = float(ms_e2e.item())
    if rank != 0:
        return
    per_kernel, b_ef = {}, 0.0
    for b in lay["buckets"]:
        kb, be = bucket_bytes(b.dims, len(b.frames), sum(b.atom_count), s=s)
        b_ef += be
        for k, v in kb.items():
            per_kernel[k] = per_kernel.get(k, 0.0) + v
    kernels = {k: {"launches": cnt[k] // args.steps, "total_ms": tot[k] / args.steps,
                   "share": tot[k] / sum(tot.values())} for k in tot}
    dom = max(tot, key=tot.get) if tot else None
    peak, peak_kind = measured_peak()
    roof = None
    for k, v in kernels.items():
        if k in per_kernel:
            v["achieved_gbs"] = per_kernel[k] / (v["total_ms"] * 1e-3) / 1e9
    if dom is not None and dom in per_kernel:
        ach = kernels[dom]["achieved_gbs"]
        roof = {"kernel": dom, "bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                "frac": ach / peak, "peak_source": f"{peak_kind} hbm_gbs", "traffic": None,
                "algorithmic_bytes_per_step": per_kernel[dom],
                "note": "rank 0's share; all launches of the kernel in one step (one per mesh bucket)"}
    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        atoms, t, threads = oracle_batch_time()
        cpu = {"value": atoms / t, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"first 120 frames of the batch ({atoms} atoms), E+F by the C/OpenMP oracle"}
    total = sum(counts)
    step_gbs = b_ef / (ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": total / (ms_max * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": args.dtype, "data": "synthetic (seeded)",
        "config": {"workload": BATCH_WORKLOAD, "frames": len(counts), "atoms": total,
                   "frames_rank0": nf_local, "atoms_rank0": N, "mesh_buckets_rank0": len(lay["buckets"]),
                   "parallelism": f"frame-dp{world} (LPT by estimated cost)" if world > 1 else "single",
                   "l2": "meshes of all frames (~1 GB per array) larger than L2"},
        "e2e": {"value": total / (ms_e2e * 1e-3), "unit": UNIT, "ms_per_step": ms_e2e,
                "h2d_bytes_per_step": N * 4 * s, "d2h_bytes_per_step": nf_local * s + N * 3 * s},
        "roofline": roof,
        "step_roofline": {"algorithmic_bytes": b_ef, "achieved": step_gbs, "peak": peak, "unit": "GB/s",
                          "frac": step_gbs / peak},
        "kernels": kernels,
        "gpu_launches": int(launches),
        "host_enqueue_ms_per_step": host_ms,
        "clocks": clk,
        "cpu_baseline": cpu,
        "energy_sum_rank0": e_sum,
    }
    print(json.dumps(line), flush=True)


def run_gpu(args, rank: int, world: int):
    import numpy as np
    import torch
    import torch.distributed as dist

    from sog_b200 import Sog, _lib

    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    cfg = workload(args.config)
    dt = torch.float64 if args.dtype == "f64" else torch.float32
    slab = world > 1 and args.mode == "slab"
    # slab: every rank holds the same system and its mesh is split over the
    # ranks; frames: every rank solves its own system (seeded by rank)
    r, q, cell, amp_raw, bw = make_inputs(cfg, seed=0 if slab else rank)
    dims = mesh_dims(cfg)
    N = cfg["natoms"]
    transport = args.transport

    def build_model(tr):
        return Sog({"use_atomwise": False, "use_bspline_fft": True, "bspline_order": cfg["order"],
                    "n_dl": cfg["n_dl"], "amp": torch.tensor(amp_raw, dtype=dt),
                    "bandwidth": torch.tensor(bw, dtype=dt), "trainable_kernel": False,
                    "mesh_decomposition": "slab" if slab else "none",
                    "slab_transport": tr}).to(dev)

    model = build_model(transport)
    gauss = model.gaussian
    r_d = torch.tensor(r, dtype=dt, device=dev)
    q_d = torch.tensor(q, dtype=dt, device=dev)
    cell_d = torch.tensor(cell[None], dtype=dt, device=dev)

    def barrier():
        if world > 1:
            dist.barrier()

    def align_streams():
        # after the host barrier the ranks leave at slightly different times;
        # a one-element sum enqueued right before the first event lines up
        # the GPUs' streams themselves, so the first timed step does not
        # absorb the host-side release skew
        if world > 1:
            dist.all_reduce(torch.zeros(1, device=dev))

    def step_device():
        return gauss.compute_bundle(q=q_d, r=r_d, cell=cell_d, compute_force=True)

    # warm-up (every rank fails the same way when peer memory is unavailable:
    # the library agrees on it collectively, so all fall back together)
    try:
        step_device()
    except _lib.SogError as exc:
        if not (slab and transport == "peer" and "peer memory" in str(exc)):
            raise
        print(f"rank {rank}: peer transport unavailable ({exc}); using the exchange transport",
              file=sys.stderr, flush=True)
        transport = "exchange"
        model = build_model(transport)
        gauss = model.gaussian
        step_device()
    for _ in range(args.warmup - 1):
        step_device()
    torch.cuda.synchronize()
    plan = next(p for p in _lib.PLANS.plans.values() if p.key[4] == dims)

    # ---- device-resident timed region ----
    # Without a collective inside the step (one GPU, or independent systems
    # per rank) the K steps are captured into one CUDA graph and replayed as
    # the timed region: the host enqueues them at once, so a pause of the
    # launching thread cannot leave the GPU idle between steps.  The slab
    # step calls NCCL between its kernels and is launched eagerly.
    stream = torch.cuda.current_stream()
    graph = None
    if not slab and not args.eager:
        plan.set_timing(True, events=48 * args.steps + 64)
        l0 = _lib.launch_count()
        graph = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(graph):
                for _ in range(args.steps):
                    out = step_device()
            launches = _lib.launch_count() - l0
            graph.replay()                   # upload; one untimed pass
            torch.cuda.synchronize()
        except Exception as exc:             # fall back to eager launches
            print(f"rank {rank}: CUDA graph capture failed ({exc}); timing eager launches",
                  file=sys.stderr, flush=True)
            graph = None
            torch.cuda.synchronize()
    if graph is None:
        plan.set_timing(True)
    # every rank starts its clock sampler first; the barrier right before the
    # first event then lines the ranks up, so no rank's sampler start-up
    # lands inside another rank's first timed step
    clocks = ClockSampler(local)
    clocks.start()
    time.sleep(0.3)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
    gc.collect()
    gc.disable()          # no collector pause inside the timed steps
    barrier()
    torch.cuda.synchronize()
    align_streams()
    if graph is not None:
        ev0.record(stream)
        h0 = time.perf_counter()
        graph.replay()
        host_ms = (time.perf_counter() - h0) * 1e3 / args.steps
        ev1.record(stream)
    else:
        l0 = _lib.launch_count()
        ev0.record(stream)
        marks[0].record(stream)
        h0 = time.perf_counter()
        for i in range(args.steps):
            out = step_device()
            marks[i + 1].record(stream)
        host_ms = (time.perf_counter() - h0) * 1e3 / args.steps   # enqueue time per step
        ev1.record(stream)
    torch.cuda.synchronize()
    gc.enable()
    if graph is None:
        launches = _lib.launch_count() - l0
        step_ms = [marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)]
    clk = clocks.stop()
    barrier()
    ms = ev0.elapsed_time(ev1) / args.steps
    kt = plan.timings()
    plan.set_timing(False)
    graph_used = graph is not None
    if graph is not None:
        # per-step device time from the kernels of each call (the first kernel
        # of a call is its frame set-up)
        step_ms, acc = [], None
        for name, t in kt:
            if name == "frame_setup":
                if acc is not None:
                    step_ms.append(acc)
                acc = 0.0
            acc = (acc or 0.0) + t
        if acc is not None:
            step_ms.append(acc)
    ms_all = torch.tensor([ms], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_all, op=dist.ReduceOp.MAX)
    ms_max = float(ms_all.item())
    energy0 = float(out["energy"][0])

    # ---- end-to-end through the public API with host buffers ----
    r_h = torch.tensor(r, dtype=dt).pin_memory()
    q_h = torch.tensor(q, dtype=dt).pin_memory()
    e_h = torch.empty(1, dtype=dt).pin_memory()
    f_h = torch.empty(N, 3, dtype=dt).pin_memory()
    r_in = torch.empty(N, 3, dtype=dt, device=dev)
    q_in = torch.empty(N, dtype=dt, device=dev)

    def step_e2e():
        r_in.copy_(r_h, non_blocking=True)
        q_in.copy_(q_h, non_blocking=True)
        o = model(positions=r_in, cell=cell_d, latent_charges=q_in, compute_force=True)
        e_h.copy_(o["E_lr"], non_blocking=True)
        f_h.copy_(o["forces"], non_blocking=True)

    for _ in range(max(1, args.warmup)):
        step_e2e()
    torch.cuda.synchronize()
    g_e2e = None
    if graph is not None:
        del graph                      # its memory pool is no longer needed
        g_e2e = torch.cuda.CUDAGraph()
        try:
            with torch.cuda.graph(g_e2e):
                for _ in range(args.steps):
                    step_e2e()
            g_e2e.replay()
            torch.cuda.synchronize()
        except Exception as exc:
            print(f"rank {rank}: CUDA graph capture of the e2e step failed ({exc})", file=sys.stderr,
                  flush=True)
            g_e2e = None
            torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    if g_e2e is not None:
        g_e2e.replay()
    else:
        for _ in range(args.steps):
            step_e2e()
    e1.record(stream)
    torch.cuda.synchronize()
    ms_e2e = torch.tensor([e0.elapsed_time(e1) / args.steps], dtype=torch.float64, device=dev)
    if world > 1:
        dist.all_reduce(ms_e2e, op=dist.ReduceOp.MAX)
    ms_e2e = float(ms_e2e.item())

    # per-rank kernel tables (ms per step), gathered to rank 0 (every rank
    # takes part in the same collective)
    tot, cnt = {}, {}
    for name, t in kt:
        tot[name] = tot.get(name, 0.0) + t
        cnt[name] = cnt.get(name, 0) + 1
    by_rank = None
    if world > 1:
        by_rank = [None] * world
        dist.all_gather_object(by_rank, {k: round(v / args.steps, 4) for k, v in tot.items()})

    # ---- one evaluation of the 1/8-scale sample checked against the oracle
    # (outside the timed region; N = 1 only, like the CPU baseline) ----
    cpu = parity = None
    if world == 1 and not args.no_cpu_baseline:
        ccfg, times, threads, oref = oracle_eval_time("cfg5_eighth", reps=3, warm=1)
        tmed = statistics.median(times)
        cpu = {"value": ccfg["natoms"] / tmed, "unit": UNIT, "cores": threads, "kind": "port",
               "sample": f"{ccfg['workload']}; C/OpenMP oracle E+F, median of 3 after 1 warm-up, "
                         f"{tmed:.2f} s per evaluation"}
        rr, qq, cc, ampr, bwr = make_inputs(ccfg, 0)
        g8 = Sog({"use_atomwise": False, "use_bspline_fft": True, "bspline_order": ccfg["order"],
                  "n_dl": ccfg["n_dl"], "amp": torch.tensor(ampr, dtype=dt),
                  "bandwidth": torch.tensor(bwr, dtype=dt), "trainable_kernel": False}).to(dev).gaussian
        o8 = g8.compute_bundle(q=torch.tensor(qq, dtype=dt, device=dev),
                               r=torch.tensor(rr, dtype=dt, device=dev),
                               cell=torch.tensor(cc[None], dtype=dt, device=dev), compute_force=True)
        e8 = float(o8["energy"][0])
        f8 = o8["forces"].double().cpu().numpy()
        fmax = float(np.abs(oref["forces"]).max())
        parity = {"sample": ccfg["workload"], "against": "oracle (C/OpenMP, fp64)",
                  "energy_rel_err": abs(e8 - oref["energy"]) / abs(oref["energy"]),
                  "force_max_abs_err": float(np.abs(f8 - oref["forces"]).max()),
                  "force_max_rel_err": float(np.abs(f8 - oref["forces"]).max()) / fmax,
                  "tolerance": ("energy rel 1e-10, force max-abs 1e-9" if dt == torch.float64
                                else "energy rel 1e-5, force max-abs / max |F| 1e-5")}
        del o8, g8

    if rank != 0:
        return
    # ---- roofline of the dominant kernel (the one with the largest stream
    # time among those that move mesh arrays; barriers and NCCL sums are
    # reported in the kernel table but carry no algorithmic bytes) ----
    s = 8 if dt == torch.float64 else 4
    b_ef, per_kernel = algorithmic_bytes(cfg, s=s, parts=world if slab else 1)
    kernels = {k: {"launches": cnt[k], "total_ms": tot[k], "avg_ms": tot[k] / cnt[k],
                   "share": tot[k] / sum(tot.values())} for k in tot}
    work = {k: v for k, v in tot.items() if k in per_kernel}
    dom = max(work, key=work.get) if work else None
    top = max(tot, key=tot.get) if tot else None
    peak, peak_kind = measured_peak()
    roof = None
    if dom is not None:
        ach = per_kernel[dom] / (kernels[dom]["avg_ms"] * 1e-3) / 1e9
        traffic = profiled_traffic(dom, args.config)
        if traffic is not None and slab:
            traffic /= world
        roof = {"kernel": dom, "bound": "hbm", "achieved": ach, "peak": peak, "unit": "GB/s",
                "frac": ach / peak, "peak_source": f"{peak_kind} hbm_gbs",
                "traffic": traffic,
                "traffic_source": (f"ncu capture committed in profiles/{TRAFFIC_PROFILE} (one launch "
                                   "of this kernel on the quarter-size 256x256x512 case, scaled to this "
                                   "size by its algorithmic bytes; not measured in this run)"
                                   if traffic is not None else None),
                "algorithmic_bytes_per_launch": per_kernel[dom],
                "largest_stream_time": {"name": top, "share": kernels[top]["share"]}}
    for k, v in kernels.items():
        if k in per_kernel:
            v["achieved_gbs"] = per_kernel[k] / (v["avg_ms"] * 1e-3) / 1e9
    step_gbs = b_ef / (ms * 1e-3) / 1e9
    systems = 1 if slab else world      # systems evaluated per step by the whole job
    nvlink = None
    if slab:
        # bytes each rank sends per evaluation: (P-1)/P of its spectrum share
        # forward and of its three field shares back, plus the halo planes
        nx, ny, nz = dims
        share = (nz // world) * ny * (nx // 2 + 1) * 2 * s
        sent = (share + 3 * share) * (world - 1) / world + (cfg["order"] - 1) * nx * ny * 3 * s
        ex_ms = sum(v["total_ms"] for k, v in kernels.items()
                    if k.startswith("exchange") or k.startswith("barrier")) / args.steps
        if transport == "peer":
            # the stores travel inside these kernels: their stream time bounds
            # the link time from above, so the rate is a lower bound
            storing = ("fft_y_fwd", "zfused", "halo_push")
            st_ms = sum(kernels[k]["total_ms"] for k in storing if k in kernels) / args.steps
            ach_nv = sent / (st_ms * 1e-3) / 1e9 if st_ms > 0 else None
            note = ("peer: the transposes are stored into the other GPUs' buffers by the y-FFT and "
                    "fused z kernels (and the halo by halo_push); achieved = bytes sent per rank / "
                    "those kernels' stream time per step (they compute too, so a lower bound); "
                    "exchange_ms is the stream time of the barriers and sums")
        else:
            st_ms = ex_ms
            ach_nv = sent / (ex_ms * 1e-3) / 1e9 if ex_ms > 0 else None
            note = "exchange time is the stream time of the NCCL calls (all-to-all, halo, sums)"
        nvlink = {"bytes_per_rank_per_step": sent, "exchange_ms_per_step": ex_ms,
                  "storing_ms_per_step": st_ms, "achieved_gbs": ach_nv,
                  "frac": ach_nv / 770.0 if ach_nv else None,
                  "peak": 770.0, "unit": "GB/s", "peak_source": "measured peer copy per direction",
                  "transport": transport, "note": note}
    if slab:
        parallelism = (f"slab{world} (z slabs; transposes stored by the FFT kernels into peer GPUs' "
                       "buffers over NVLink, NCCL sums as barriers)" if transport == "peer" else
                       f"slab{world} (z slabs, NCCL all-to-all transposes)")
    else:
        parallelism = f"frame-dp{world}" if world > 1 else "single"
    line = {
        "metric": METRIC, "value": systems * N / (ms_max * 1e-3), "unit": UNIT, "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms_max, "higher_is_better": True,
        "scaling": "strong" if slab else "weak", "vs_baseline": None, "dtype": args.dtype,
        "data": "synthetic (seeded)",
        "config": {"workload": cfg["workload"], "atoms_per_gpu": N // world if slab else N,
                   "mesh": list(dims), "spline": f"bspline{cfg['order']}", "gaussians": cfg["m"],
                   "parallelism": parallelism,
                   "l2": "inputs and mesh arrays larger than L2 (>= 1 GB each)"},
        "e2e": {"value": systems * N / (ms_e2e * 1e-3), "unit": UNIT, "ms_per_step": ms_e2e,
                "h2d_bytes_per_step": N * 4 * s, "d2h_bytes_per_step": s + N * 3 * s},
        "roofline": roof,
        "nvlink": nvlink,
        "step_roofline": {"algorithmic_bytes": b_ef, "achieved": step_gbs, "peak": peak,
                          "unit": "GB/s", "frac": step_gbs / peak},
        "kernels": kernels,
        "gpu_launches": int(launches),
        "host_enqueue_ms_per_step": host_ms,
        "cuda_graph": {"device": graph_used, "e2e": g_e2e is not None},
        "step_ms": [round(x, 4) for x in step_ms],
        "clocks": clk,
        "cpu_baseline": cpu,
        "parity": parity,
        "energy_frame0": energy0,
    }
    if by_rank is not None:
        line["kernels_ms_per_step_by_rank"] = by_rank
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="sog_b200", choices=["sog_b200", "reference"])
    ap.add_argument("--config", default="cfg5", choices=["cfg5", "cfg5_eighth", "cfg5_quarter", "cfg5_zslab", "cfg2", "cfg4"])
    ap.add_argument("--dtype", default="f64", choices=["f64", "f32"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--transport", default="peer", choices=["peer", "exchange"],
                    help="slab mode: NVLink stores from the FFT kernels (peer) or NCCL all-to-all")
    ap.add_argument("--eager", action="store_true",
                    help="launch the timed steps one by one instead of replaying a CUDA graph")
    ap.add_argument("--mode", default="slab", choices=["slab", "frames"],
                    help="N>1: split one system's mesh over the GPUs (slab) or give each GPU "
                         "its own system (frames)")
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    if args.impl == "reference":
        run_reference(args, rank)
        return
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", "0")))
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    try:
        if args.config == "cfg4":
            run_gpu_batch(args, rank, world)
        else:
            run_gpu(args, rank, world)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
