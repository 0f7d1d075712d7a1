"""Benchmark: fwd+bwd rays/s of the Voronoi-foam tracer on synthetic foams.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config surface|unbounded|medium|tiny|densify]
    python bench.py --impl reference ...     # the CPU restatement of the reference path

One step = one pass of the hot path over one batch of rays (the headline:
the 4M-site surface foam, 8,388,608 rays): the sdfnet MLP at every site
(whose output is the sites' SDF), cell-record build, forward walk, backward
walk (NeuS mode, fp32, SH degree 3, inv_s = 50, weight_threshold 1e-7,
contributions on), the MLP's backward, and with N > 1 GPUs the NCCL
all-reduce of the gradients.  Rays are sharded across ranks (each rank
traces its own batches; the foam is replicated), so per-GPU work is fixed:
weak scaling.  Rank 0 prints one JSON line: the device-timed value, the
end-to-end value through TraceRays with host copies (`e2e`), the roofline of
the dominant kernel, the CPU baseline on a bounded sample and the GPU's
parity against it on that sample.  Component timings for profiling:
--mlp-layer, --mlp-step, --eikonal.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "fwd+bwd rays/sec at 4M-site foam, 1/2/4/8 B200; % of HBM roofline"
UNIT = "rays/s"
INV_S = 50.0
# library kernels of the fused sdfnet per step: encode, 8 hidden layers (the
# last with the output layer), 8 dgrads, 9 weight gradients, the encoding's
# gradient, decode
MLP_LAUNCHES = 28
MLP_SEED = 11  # the surface config's sdfnet (Xavier init) that produces the sites' SDF
FALLBACK_HBM_GBS = 6650.0

CONFIGS = {
    # name: (synthetic config, rays per step)
    "surface": ("surface", 8 << 20),
    "medium": ("medium", 5_120_000),
    "unbounded": ("unbounded", 8 << 20),
    "tiny": ("tiny", 16384),
}
# max_intersections per config (the reference's default 1024; 4096 for the
# unbounded scene's long rays)
MAX_STEPS = {"unbounded": 4096}


def log(*a):
    print(*a, file=sys.stderr, flush=True)


# --------------------------------------------------------------------------
# workload
# --------------------------------------------------------------------------

CACHE_DIR = os.environ.get("SDFOAM_BENCH_CACHE", os.path.join(tempfile.gettempdir(), "sdfoam_b200_scenes"))


def gpu_adjacency(points: np.ndarray):
    """Delaunay CSR of the (sorted) sites from the library's GPU rebuild, the
    same bits as Qhull's (checked against it up to 4M sites in the tests)."""
    import torch
    from sdfoam_b200.triangulation import delaunay_adjacency
    adj, off = delaunay_adjacency(torch.from_numpy(np.ascontiguousarray(points)).cuda())
    return adj.cpu().numpy(), off.cpu().numpy()


def load_foam(config: str, gpu: bool = True):
    """The seeded synthetic foam of a config.  Its Delaunay adjacency comes
    from the GPU rebuild (12 s at 4M sites), or from scipy's Qhull on the host
    for the reference arm, which runs none of this library's kernels (two
    minutes at 4M sites; the same bits).  The finished foam is cached on local
    disk and shared by every process of one machine; with several ranks,
    rank 0 builds it and the others wait for the file."""
    from sdfoam_b200 import synthetic as syn
    os.makedirs(CACHE_DIR, exist_ok=True)
    path = os.path.join(CACHE_DIR, f"{config}_v1.npz")
    rank = int(os.environ.get("RANK", "0"))
    if not os.path.exists(path):
        if rank == 0:
            t = time.time()
            foam = syn.make_foam(config, adjacency_fn=gpu_adjacency) if gpu else syn.make_foam(config)
            tmp = path + f".tmp{os.getpid()}.npz"
            np.savez(tmp, points=foam.points, attributes=foam.attributes, adjacency=foam.adjacency,
                     offsets=foam.offsets, sdf=foam.sdf, sh_degree=foam.sh_degree)
            os.replace(tmp, path)
            log(f"[bench] built foam {config} in {time.time() - t:.1f}s")
        else:
            t = time.time()
            while not os.path.exists(path):
                if time.time() - t > 1800:
                    raise RuntimeError("timed out waiting for rank 0 to build the foam")
                time.sleep(2.0)
    z = np.load(path)
    return syn.Foam(z["points"], z["attributes"], z["adjacency"], z["offsets"], z["sdf"], int(z["sh_degree"]))


RAY_ORDERS = {"tiles": "view-major, 8x4 pixel tiles",
              "shuffled": "shuffled: a seeded permutation of all views' rays (training's order)"}


def build_workload(config: str, batch: int, max_rays: int | None = None, gpu: bool = True, order: str = "tiles"):
    from sdfoam_b200 import synthetic as syn
    t = time.time()
    foam = load_foam(config, gpu)
    log(f"[bench] foam {config}: {foam.points.shape[0]} sites, {foam.adjacency.shape[0]} CSR entries "
        f"({time.time() - t:.1f}s)")
    cams = syn.views(config)
    rays, start = syn.camera_rays(foam, cams, tile=(8, 4))
    if order == "shuffled":
        # the order training draws rays in (random rays of random images)
        perm = np.random.default_rng(17).permutation(rays.shape[0])
        rays, start = rays[perm], start[perm]
    if max_rays is not None:
        rays, start = rays[:max_rays], start[:max_rays]
    nb = max(1, rays.shape[0] // batch) if rays.shape[0] >= batch else 1
    grad = np.random.default_rng(7).normal(0.0, 1.0, (min(batch, rays.shape[0]), 4)).astype(np.float32)
    return foam, rays, start, grad, nb, len(cams)


def bytes_model(steps: int, rays: int, dbar: float, replay_steps: float = 0.0):
    """Algorithmic bytes of the reference layout (fp32, SH 3): per walk step
    forward 232 + 8 d (offsets 8, diffs 8 d, id 4, next site 12, attributes
    196, alpha 4, contribution 8), backward 636 + 8 d (the same reads plus SH
    gradient RMW 384, SDF gradient 8, point gradient 24); per ray forward 48,
    backward 60 bytes.  With the exit record, the forward also writes one byte
    per recorded step and a backward step that replays it reads one face's
    diff and that byte instead of the whole row's diffs (8 + 1 for 8 d)."""
    fwd = steps * (232.0 + 8.0 * dbar) + replay_steps * 1.0 + rays * 48.0
    bwd = steps * (636.0 + 8.0 * dbar) - replay_steps * (8.0 * dbar - 9.0) + rays * 60.0
    return fwd, bwd


def hbm_peak():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            v = float(json.load(f)["hbm_gbs"])
        return v, "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def ncu_value(name: str, key: str):
    """A figure from a committed ncu summary (profiles/<name>.txt, a line
    '<key>=<number>'), or None."""
    p = os.path.join(ROOT, "profiles", name + ".txt")
    try:
        for line in open(p):
            if line.startswith(key + "="):
                return float(line.split("=", 1)[1])
    except (OSError, ValueError):
        pass
    return None


def ncu_traffic(name: str):
    """Per-launch DRAM bytes of a kernel at the bench's full launch size
    (line 'dram_bytes_per_launch_full=<bytes>')."""
    return ncu_value(name, "dram_bytes_per_launch_full")


LIMITER_KEYS = ("l1tex_throughput_pct", "l2_throughput_pct", "dram_throughput_pct", "issue_active_pct",
                "warps_active_pct", "long_scoreboard_per_issue")


def roofline(dom, dom_bytes, dom_ms, fwd_b, bwd_b, k_fwd, k_bwd, args):
    """Roofline of the dominant walk kernel.  `achieved` is the DRAM traffic
    of one launch (ncu dram__bytes_read.sum + dram__bytes_write.sum of the
    same workload, profiles/trace_<kernel>_<config>.txt) over its CUDA-event
    time: the walk re-reads each cell from L1 / L2 for the coherent rays of a
    warp, so HBM runs at a few per cent of its peak and the kernel is bound
    by the L1 data pipeline and dependent-load latency, whose ncu figures are
    in `limiter`.  `algorithmic_gbs` is the survey's per-step byte model of
    the reference layout over the same time (a logical figure that counts
    cache hits, which is why it can exceed the HBM peak)."""
    peak, peak_kind = hbm_peak()
    name = f"trace_{dom}_{args.config}"
    traffic = ncu_traffic(name) if args.ray_order == "tiles" and not args.sort_rays else None
    algo = dom_bytes / (dom_ms / 1000.0) / 1e9
    walk_algo = (fwd_b + bwd_b) / ((k_fwd + k_bwd) / 1000.0) / 1e9
    achieved = traffic / (dom_ms / 1000.0) / 1e9 if traffic else algo
    lim = {k: ncu_value(name, k) for k in LIMITER_KEYS}
    lim = {k: v for k, v in lim.items() if v is not None}
    if lim:
        lim["source"] = f"profiles/{name}.txt (ncu --set full of one launch on the first 1M rays)"
    return {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
            "traffic": traffic, "kernel": f"{dom} walk",
            "achieved_basis": ("ncu DRAM bytes per launch / CUDA-event launch time" if traffic else
                               "algorithmic bytes (no ncu capture of this workload)"),
            "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
            else "fallback 6.65 TB/s",
            "algorithmic_bytes_per_launch": dom_bytes, "algorithmic_gbs": algo, "algorithmic_frac": algo / peak,
            "limiter": lim or None,
            "walk_fwd_bwd": {"algorithmic_gbs": walk_algo, "algorithmic_frac": walk_algo / peak}}


class ClockSampler:
    """nvidia-smi clock / throttle-reason samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200"], stdout=self.file, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        if self.proc is None or self.file is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        try:
            with open(self.file.name) as f:
                for line in f:
                    parts = [x.strip() for x in line.split(",")]
                    if len(parts) >= 9:
                        rows.append(parts)
            os.unlink(self.file.name)
        except OSError:
            pass
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower().startswith("active")})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# --------------------------------------------------------------------------
# CPU leg (the reference path restated on host cores)
# --------------------------------------------------------------------------

def make_mlp(foam, dtype):
    """The surface config's sdfnet: the reference architecture, Xavier init
    drawn from a seeded generator (the same weights for every dtype)."""
    import torch
    from sdfoam_b200.sdfnet import SDFNetwork
    gen = torch.Generator().manual_seed(MLP_SEED)
    return SDFNetwork(d_hidden=256, n_layers=8, multires=6, init="xavier", dtype=dtype, point_cloud=foam.points,
                      generator=gen)


SDF_SOURCE_REF = {"surface": "sdfnet (Xavier init, seed 11) evaluated in float32 PyTorch layers on the host"}
SDF_SOURCE_GPU = {"surface": "sdfnet (Xavier init, seed 11) evaluated by the fused bf16 tcgen05 path on the GPU"}


def with_mlp_sdf(foam, config: str):
    """The walk workload of the surface config: the sites' SDF channel is the
    sdfnet's output, as in the training step (dense gradient rows along the
    whole ray).  Host-side evaluation for the reference arm, which runs none
    of this library's kernels: the same network in plain float32 PyTorch
    layers, cached per machine.  (The GPU arm evaluates it with the fused
    bf16 path; the two SDFs agree to bf16 rounding.)"""
    from dataclasses import replace
    if config != "surface":
        return foam
    path = os.path.join(CACHE_DIR, f"{config}_sdf_xavier{MLP_SEED}.npy")
    if os.path.exists(path):
        sdf = np.load(path)
    else:
        import torch
        mlp = make_mlp(foam, torch.float32)
        pts = torch.from_numpy(foam.points)
        with torch.no_grad():
            sdf = torch.cat([mlp.forward_layers(pts[i:i + 262144])[:, 0]
                             for i in range(0, pts.shape[0], 262144)]).numpy().astype(np.float32)
        tmp = path + f".tmp{os.getpid()}.npy"
        np.save(tmp, sdf)
        os.replace(tmp, path)
    att = foam.attributes.copy()
    att[:, -1] = sdf
    return replace(foam, attributes=att)


def oracle_scene(foam):
    from oracle import oracle as orc
    return orc.OracleScene(foam.points, foam.attributes, foam.adjacency, foam.offsets, foam.sh_degree)


def cpu_trace(sc, rays, start, grad, max_rays: int, threads: int, inv_s: float = INV_S, max_steps: int = 1024):
    """The CPU restatement's forward + backward over the first max_rays rays
    (timed): (rays/s, rays, seconds, forward outputs)."""
    from oracle import oracle as orc
    st = orc.settings(neus=True, sharpness=inv_s, max_intersections=max_steps)
    n = min(max_rays, rays.shape[0])
    r, s, g = rays[:n], start[:n], grad[:n]
    t = time.perf_counter()
    fw = orc.trace_forward(sc, st, r, s, threads=threads)
    orc.trace_backward(sc, st, r, s, fw["rgba"], g, threads=threads)
    dt = time.perf_counter() - t
    return n / dt, n, dt, fw


def sample_parity(sc, rays, start, grad, fw_ref, gpu, threads: int, inv_s: float = INV_S, max_steps: int = 1024):
    """Compares the GPU's outputs on the CPU sample (the first n rays of the
    benchmarked batch, same attributes) with the CPU restatement's:
    hit counts bit for bit, rgba within 1e-4 relative (floor 1e-6),
    contributions within 1e-4, gradients within 1e-3 relative with an absolute
    floor of 3e-5 x the sum of |terms| accumulated into the entry (both sides
    sum float atomics in their own order).  Also counts the rays whose
    termination could fall on another step under the reference's __expf
    (oracle exp_interval)."""
    from oracle import oracle as orc
    st = orc.settings(neus=True, sharpness=inv_s, max_intersections=max_steps)
    n = rays.shape[0]
    amb = orc.trace_forward(sc, st, rays, start, return_contribution=False, threads=threads, ambiguity=True)
    rb = orc.trace_backward(sc, st, rays, start, fw_ref["rgba"], grad, threads=threads, with_abs=True)
    hits = np.asarray(gpu["num_intersections"]).reshape(-1)
    same = hits == fw_ref["num_intersections"]
    rg = np.asarray(gpu["rgba"], np.float64)
    rr = fw_ref["rgba"].astype(np.float64)
    tol = 1e-4 * np.abs(rr) + 1e-6
    rgba_ok = np.abs(rg - rr) <= tol
    cg = np.asarray(gpu["contribution"], np.float64).reshape(-1)
    cr = fw_ref["contribution"].astype(np.float64)
    con_ok = np.abs(cg - cr) <= 1e-4 * np.abs(cr) + 1e-6

    def grads_ok(a, b, babs):
        a = np.asarray(a, np.float64)
        b = np.asarray(b, np.float64)
        return np.abs(a - b) <= 1e-3 * np.abs(b) + 3e-5 * np.asarray(babs, np.float64) + 1e-7

    ag = grads_ok(gpu["attr_grad"], rb["attr_grad"], rb["attr_grad_abs"])
    pg = grads_ok(gpu["points_grad"], rb["points_grad"], rb["points_grad_abs"])
    sg, sr = float(gpu["sharpness_grad"]), float(rb["sharpness_grad"][0])
    return {
        "sample": f"first {n} rays of the benchmarked batch, same attributes (SDF from the GPU sdfnet), "
                  f"GPU (C ABI) vs the CPU restatement oracle/sdfoam_oracle.c",
        "rays": int(n), "walk_steps": int(fw_ref["num_intersections"].astype(np.int64).sum()),
        "hit_counts_bit_exact": float(same.mean()),
        "rgba_within_1e-4": float(rgba_ok.mean()), "rgba_max_err_over_tol": float((np.abs(rg - rr) / tol).max()),
        "rgba_bit_identical": float((np.asarray(gpu["rgba"], np.float32).view(np.uint32)
                                     == fw_ref["rgba"].view(np.uint32)).mean()),
        "contribution_within_1e-4": float(con_ok.mean()),
        "attr_grad_within_1e-3": float(ag.mean()), "points_grad_within_1e-3": float(pg.mean()),
        "sharpness_grad_rel_err": abs(sg - sr) / max(abs(sr), 1e-30),
        "threshold_ambiguous_rays": int(amb["ambiguous"].sum()),
        "threshold_ambiguous_frac": float(amb["ambiguous"].mean()),
        "pass": bool(same.all() and rgba_ok.all() and con_ok.all() and ag.all() and pg.all()
                     and abs(sg - sr) <= 1e-3 * abs(sr) + 1e-4),
    }


def cells_gb(num_points: int, csr_entries: int) -> float:
    """Size of the walk's cell records (site records 256 B, face records 16 B,
    plane slots 8 B; SH degree 3)."""
    return (num_points * 256 + csr_entries * 16 + (csr_entries + 3 * num_points + 8) * 8) / 1e9


def workload_config(args, foam, batch: int, nviews: int, world: int = 1) -> dict:
    """The `config` object of both arms' lines (identical for the same run)."""
    n = int(foam.points.shape[0])
    e = int(foam.adjacency.shape[0])
    return {"workload": args.config, "sites": n, "csr_entries": e, "rays_per_step_per_gpu": int(batch),
            "views": nviews, "sh_degree": 3, "mode": "neus", "inv_s": args.inv_s, "max_intersections": MAX_STEPS.get(
                args.config, 1024), "ray_order": RAY_ORDERS[args.ray_order],
            "l2": ("inputs larger than L2 (cell records %.2f GB)" if cells_gb(n, e) > 0.126 else
                   "inputs smaller than L2 (cell records %.2f GB; a component case, not the headline)") % cells_gb(n, e),
            "parallelism": f"rays sharded over {world} GPU(s), foam replicated"}


def run_reference(args):
    """The reference path's CPU restatement on the host cores: every step
    traces the same bounded sample (the first --ref-rays rays of the batch)
    forward and backward, so that ms_per_step is the time of what ran; the
    GPU arm's cpu_baseline times the same sample."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    cfg, batch = CONFIGS[args.config]
    foam, rays, start, grad, nb, nviews = build_workload(cfg, batch, gpu=False, order=args.ray_order)
    foam = with_mlp_sdf(foam, args.config)
    threads = os.cpu_count() or 1
    sample = min(args.ref_rays, batch, rays.shape[0])
    sc = oracle_scene(foam)
    for _ in range(args.warmup):
        cpu_trace(sc, rays, start, grad, min(sample, 4096), threads, args.inv_s, MAX_STEPS.get(args.config, 1024))
    times = []
    for _ in range(args.steps):
        _, n, dt, _ = cpu_trace(sc, rays, start, grad, sample, threads, args.inv_s, MAX_STEPS.get(args.config, 1024))
        times.append(dt)
    value = sample * len(times) / sum(times)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, foam, batch, nviews),
        "cpu_baseline": {"value": value, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"first {sample} rays of the {batch}-ray batch each step, fwd+bwd, CPU restatement "
                                   f"of the reference walk (oracle/sdfoam_oracle.c, OpenMP); the reference itself "
                                   f"cannot be built (Eigen and GL headers absent)"},
        "sdf_source": SDF_SOURCE_REF.get(args.config, "synthetic"),
        "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# --------------------------------------------------------------------------
# GPU leg
# --------------------------------------------------------------------------

def run_gpu(args):
    import torch
    import torch.distributed as dist

    import sdfoam_b200 as sdfoam
    from sdfoam_b200.distributed import OverlappedAllReduce, allreduce_grads, shard_batches, sharded_rows
    from sdfoam_b200.distributed import max_over_ranks as max_over_ranks_
    from sdfoam_b200.render import TraceRays

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        # NCCL prints a version banner on stdout when the communicator comes
        # up; keep stdout for the one JSON line by sending fd 1 to stderr
        # until the first collective has run.
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)

    cfg, batch = CONFIGS[args.config]
    if args.batch:
        batch = args.batch
    foam, rays, start, grad, nb, nviews = build_workload(cfg, batch, order=args.ray_order)
    N = foam.points.shape[0]
    batch = min(batch, rays.shape[0])
    pipe = sdfoam.create_pipeline(3, "float32")
    pipe.sort_rays = bool(args.sort_rays)
    pipe.max_intersections = MAX_STEPS.get(args.config)
    from sdfoam_b200.render import coherent_order
    pts = torch.from_numpy(foam.points).to(dev)
    att = torch.from_numpy(foam.attributes).to(dev)
    adj = torch.from_numpy(foam.adjacency).to(dev)
    off = torch.from_numpy(foam.offsets).to(dev)
    inv_s = torch.full((N, 1), args.inv_s, device=dev)
    # surface config: the sites' SDF comes from the sdfnet MLP (bf16, Xavier
    # init) as in the training step, for the walk-only timing as well
    mlp = None
    if args.config == "surface":
        mlp = make_mlp(foam, torch.bfloat16).to(dev)
        with torch.no_grad():
            att = torch.cat([att[:, :48], mlp(pts).float()], 1).contiguous()
        # hand the forward's activations back to the driver (keeps a profiled
        # walk-only run at a few GB of device memory)
        torch.cuda.empty_cache()
        from dataclasses import replace
        foam_walk = replace(foam, attributes=att.cpu().numpy())
    else:
        foam_walk = foam
    # this rank's batches stay resident in HBM
    my_batches = shard_batches(nb, world, rank)
    d_rays = [torch.from_numpy(rays[b * batch:(b + 1) * batch]).to(dev) for b in my_batches]
    d_start = [torch.from_numpy(start[b * batch:(b + 1) * batch]).to(dev) for b in my_batches]
    d_grad = torch.from_numpy(grad[:batch]).to(dev)

    # walk statistics for the bytes model (untimed)
    S_list, F_list = [], []
    from sdfoam_b200.render import EXIT_RECORD_STEPS
    R_list = []
    for rr, ss in zip(d_rays, d_start):
        ft = torch.empty(rr.shape[0], dtype=torch.uint32, device=dev)
        o = pipe.trace_forward(pts, att, adj, off, rr, ss, alpha_mode="sdfoam", inv_s=inv_s, _face_tests=ft)
        nint = o["num_intersections"].to(torch.int64)
        S_list.append(int(nint.sum().item()))
        R_list.append(int(nint.clamp(max=EXIT_RECORD_STEPS).sum().item()))
        F_list.append(int(ft.to(torch.int64).sum().item()))
    S_mean = sum(S_list) / len(S_list)
    R_mean = sum(R_list) / len(R_list)
    dbar = sum(F_list) / max(1, sum(S_list))
    exit_buf = pipe.exit_record(max(r.shape[0] for r in d_rays), EXIT_RECORD_STEPS, dev)
    from sdfoam_b200.render import COLOR_RECORD_STEPS
    color_buf = pipe.color_record(max(r.shape[0] for r in d_rays), COLOR_RECORD_STEPS, dev)
    site_buf = pipe.site_record(max(r.shape[0] for r in d_rays), COLOR_RECORD_STEPS, dev)

    stream = torch.cuda.current_stream(dev)

    def sync_ranks():
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()

    def max_over_ranks(ms):
        return max_over_ranks_(ms, dev) if world > 1 else ms

    # -- 1. walk kernels alone (CUDA events around each launch) -> roofline --
    def kstep(k, timers=None):
        i = k % len(d_rays)
        rr, ss = d_rays[i], d_start[i]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(4)] if timers is not None else None
        if ev: ev[0].record(stream)
        if pipe.sort_rays:
            # the walk in coherent order, as TraceRays does with sort_rays (timed)
            perm = coherent_order(rr, ss)
            rr, ss = rr[perm], ss.view(torch.int32)[perm].view(torch.uint32)
        cells = pipe.build_cells(pts, att, adj, off)
        if ev: ev[1].record(stream)
        ex = exit_buf[:rr.shape[0]]
        full = rr.shape[0] == color_buf.shape[1]
        col, sit = (color_buf, site_buf) if full else (None, None)
        fw = pipe.trace_forward(pts, att, adj, off, rr, ss, return_contribution=True, alpha_mode="sdfoam",
                                inv_s=inv_s, cells=cells, exits=ex, colors=col, sites=sit)
        if ev: ev[2].record(stream)
        pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], d_grad[:rr.shape[0]], alpha_mode="sdfoam",
                            inv_s=inv_s, cells=cells, exits=ex, colors=col, sites=sit)
        if ev: ev[3].record(stream)
        if timers is not None:
            timers.append(ev)

    for k in range(args.warmup):
        kstep(k)
    sync_ranks()
    timers = []
    for k in range(args.steps):
        kstep(k, timers)
    sync_ranks()
    k_build = sum(e[0].elapsed_time(e[1]) for e in timers) / len(timers)
    k_fwd = sum(e[1].elapsed_time(e[2]) for e in timers) / len(timers)
    k_bwd = sum(e[2].elapsed_time(e[3]) for e in timers) / len(timers)

    # -- 2. the full step through the public op (autograd), inputs in HBM ----
    # surface config: sites' SDF from the sdfnet MLP (bf16, Xavier init) at
    # every site, attributes = [SH | SDF], TraceRays forward + backward, MLP
    # backward; with N > 1 ranks, NCCL all-reduce of every gradient.
    use_mlp = mlp is not None and not args.no_mlp
    pts_p = pts.clone().requires_grad_(True)
    inv_p = inv_s.clone().requires_grad_(True)
    if use_mlp:
        sh_p = att[:, :48].clone().requires_grad_(True)
        leaves = [pts_p, sh_p, inv_p] + list(mlp.parameters())
    else:
        att_p = att.clone().requires_grad_(True)
        leaves = [pts_p, att_p, inv_p]

    # with N > 1 ranks every leaf's gradient is all-reduced as soon as the
    # backward has produced it (the per-site gradients under the sdfnet's
    # backward), the small ones together at the end
    reducer = OverlappedAllReduce(leaves) if world > 1 else None

    def full_step(rr, ss, gg):
        if use_mlp:
            # with several ranks each site's SDF is evaluated on one rank and
            # gathered everywhere (its gradient comes back summed)
            sdf = sharded_rows(mlp, pts_p) if world > 1 else mlp(pts_p)
            attributes = torch.cat([sh_p, sdf], dim=1)
        else:
            attributes = att_p
        rgba, _, _, _, _, _ = TraceRays.apply(pipe, pts_p, attributes, adj, off, rr, ss, None, True, True,
                                              inv_p, 1e-6, 48)
        rgba.backward(gg)
        if reducer is not None:
            reducer.finish()
        for p_ in leaves:
            p_.grad = None
        return rgba

    for k in range(args.warmup):
        i = k % len(d_rays)
        full_step(d_rays[i], d_start[i], d_grad[:d_rays[i].shape[0]])
    sync_ranks()
    with ClockSampler(local) as clk:
        sync_ranks()
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        t_start.record(stream)
        for k in range(args.steps):
            i = k % len(d_rays)
            full_step(d_rays[i], d_start[i], d_grad[:d_rays[i].shape[0]])
        t_end.record(stream)
        sync_ranks()
    elapsed_ms = max_over_ranks(t_start.elapsed_time(t_end))
    rays_per_rank = sum(d_rays[k % len(d_rays)].shape[0] for k in range(args.steps))
    total_rays = rays_per_rank * world
    value = total_rays / (elapsed_ms / 1000.0)

    # the gradient all-reduce alone (the same tensors, one bucket per dtype)
    allreduce_ms = None
    if world > 1:
        gbuf = [torch.zeros_like(p_) for p_ in leaves]
        allreduce_grads(gbuf)
        sync_ranks()
        a0, a1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a0.record(stream)
        for _ in range(args.steps):
            allreduce_grads(gbuf)
        a1.record(stream)
        sync_ranks()
        allreduce_ms = max_over_ranks(a0.elapsed_time(a1) / args.steps)
        del gbuf

    mlp_ms = None
    if use_mlp:
        # MLP forward + backward alone at every site (tensor-core work)
        if reducer is not None:
            reducer.enabled = False
        for _ in range(2):
            mlp(pts_p).backward(torch.ones((N, 1), device=dev))
        sync_ranks()
        m0 = torch.cuda.Event(enable_timing=True)
        m1 = torch.cuda.Event(enable_timing=True)
        m0.record(stream)
        for _ in range(args.steps):
            mlp(pts_p).backward(torch.ones((N, 1), device=dev))
        m1.record(stream)
        sync_ranks()
        mlp_ms = m0.elapsed_time(m1) / args.steps
        for p_ in leaves:
            p_.grad = None
        if reducer is not None:
            reducer.enabled = True

    # -- 3. end to end: pinned host rays / starts / upstream grads in, rgba out
    h_rays = [torch.from_numpy(rays[b * batch:(b + 1) * batch]).pin_memory() for b in my_batches]
    h_start = [torch.from_numpy(start[b * batch:(b + 1) * batch]).pin_memory() for b in my_batches]
    h_grad = torch.from_numpy(grad[:batch]).pin_memory()
    h_out = torch.empty((batch, 4), dtype=torch.float32).pin_memory()
    h2d = d2h = 0

    # Each step's inputs are copied from pinned host memory on a copy stream
    # while the previous step computes (two device slots), and its rgba goes
    # back to the host on the copy stream while the next step computes; the
    # timed region covers every copy (the last ones are waited for before
    # its end event).
    copy_stream = torch.cuda.Stream(dev)
    nmax = max(r.shape[0] for r in h_rays)
    slots = [(torch.empty((nmax, 6), dtype=torch.float32, device=dev),
              torch.empty((nmax,), dtype=torch.uint32, device=dev),
              torch.empty((nmax, 4), dtype=torch.float32, device=dev)) for _ in range(2)]
    ready = [torch.cuda.Event() for _ in range(2)]
    free = [torch.cuda.Event() for _ in range(2)]
    done = torch.cuda.Event()

    def issue_h2d(k):
        nonlocal h2d
        i, slot = k % len(h_rays), k % 2
        n = h_rays[i].shape[0]
        with torch.cuda.stream(copy_stream):
            copy_stream.wait_event(free[slot])  # the slot's previous step has finished with it
            slots[slot][0][:n].copy_(h_rays[i], non_blocking=True)
            slots[slot][1][:n].copy_(h_start[i], non_blocking=True)
            slots[slot][2][:n].copy_(h_grad[:n], non_blocking=True)
            ready[slot].record(copy_stream)
        h2d = n * (6 * 4 + 4 + 4 * 4)
        return n

    def e2e_run(nsteps):
        nonlocal d2h
        for e in free:
            e.record(stream)
        n_next = issue_h2d(0)
        for k in range(nsteps):
            slot, n = k % 2, n_next
            if k + 1 < nsteps:
                n_next = issue_h2d(k + 1)
            stream.wait_event(ready[slot])
            rr, ss, gg = slots[slot][0][:n], slots[slot][1][:n], slots[slot][2][:n]
            rgba = full_step(rr, ss, gg).detach()
            free[slot].record(stream)
            done.record(stream)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(done)
                h_out[:n].copy_(rgba, non_blocking=True)
            rgba.record_stream(copy_stream)
            d2h = rgba.numel() * 4
        stream.wait_stream(copy_stream)

    e2e_run(max(1, args.warmup))
    sync_ranks()
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    e2e_run(args.steps)
    e1.record(stream)
    sync_ranks()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e_value = total_rays / (e2e_ms / 1000.0)

    # roofline of the dominant kernel (the backward walk) and of the walk pair
    fwd_b, bwd_b = bytes_model(S_mean, batch, dbar, R_mean)
    kernels = {"build_cells_ms": k_build, "forward_ms": k_fwd, "backward_ms": k_bwd}
    if allreduce_ms is not None:
        kernels["allreduce_ms"] = allreduce_ms
        kernels["allreduce_bytes"] = int(sum(p_.numel() * p_.element_size() for p_ in leaves))
        kernels["allreduce_note"] = ("the gradient all-reduce timed alone; in the step it overlaps the sdfnet "
                                     "backward (OverlappedAllReduce)")
    if mlp_ms is not None:
        from sdfoam_b200.sdfnet import mlp_flops_per_site
        mlp_tflops = 3 * mlp_flops_per_site(mlp) * N / (mlp_ms / 1000.0) / 1e12
        kernels.update({"mlp_fwd_bwd_ms": mlp_ms, "mlp_tflops": mlp_tflops,
                        "mlp_impl": "every GEMM on the library's tcgen05 kernels: hidden layers with fused softplus "
                                    "epilogues and TMA-stored outputs (the last one also applies the output layer), "
                                    "dgrads with the fused derivative, weight gradients reducing over the rows "
                                    "(MN-major operands), the encoding's gradient with the skip gradient added"})
    dom = "backward" if k_bwd >= k_fwd else "forward"
    dom_bytes, dom_ms = (bwd_b, k_bwd) if dom == "backward" else (fwd_b, k_fwd)

    line = None
    if rank == 0:
        cpu = parity = None
        if world == 1 and not args.no_cpu_baseline:
            # the CPU restatement on the first cpu_rays rays of the batch
            # (timed), then the GPU's outputs for the same rays against it
            threads = os.cpu_count() or 1
            max_steps = MAX_STEPS.get(args.config, 1024)
            sc = oracle_scene(foam_walk)
            rate, n, dt, fw_ref = cpu_trace(sc, rays, start, grad, args.cpu_rays, threads, args.inv_s, max_steps)
            cpu = {"value": rate, "unit": UNIT, "cores": threads, "kind": "port",
                   "sample": f"first {n} rays of the batch, fwd+bwd ({dt:.1f}s), CPU restatement of the "
                             f"reference walk (oracle/sdfoam_oracle.c, OpenMP)"}
            rr = torch.from_numpy(rays[:n]).to(dev)
            ss = torch.from_numpy(start[:n]).to(dev)
            gg = torch.from_numpy(grad[:n]).to(dev)
            ex = exit_buf[:n]
            col = pipe.color_record(n, COLOR_RECORD_STEPS, dev)
            sit = pipe.site_record(n, COLOR_RECORD_STEPS, dev)
            fw = pipe.trace_forward(pts, att, adj, off, rr, ss, return_contribution=True, alpha_mode="sdfoam",
                                    inv_s=inv_s, exits=ex, colors=col, sites=sit)
            bw = pipe.trace_backward(pts, att, adj, off, rr, ss, fw["rgba"], gg, alpha_mode="sdfoam", inv_s=inv_s,
                                     exits=ex, colors=col, sites=sit)
            del col, sit
            gpu_out = {"num_intersections": fw["num_intersections"].cpu().numpy(), "rgba": fw["rgba"].cpu().numpy(),
                       "contribution": fw["contribution"].cpu().numpy(), "attr_grad": bw["attr_grad"].cpu().numpy(),
                       "points_grad": bw["points_grad"].cpu().numpy(),
                       "sharpness_grad": float(bw["sharpness_grad"].sum().item())}
            parity = sample_parity(sc, rays[:n], start[:n], grad[:n], fw_ref, gpu_out, threads, args.inv_s,
                                   max_steps)
            del sc, fw_ref, gpu_out, fw, bw
        # ours: cell build (sites, faces), forward walk, backward (walk, fold);
        # the fused MLP adds encode, 8 activate, 8 deactivate and decode
        launches_per_step = 2 + 1 + 2 + (MLP_LAUNCHES if use_mlp and mlp.fused_ok(pts_p) else 0)
        cfgd = workload_config(args, foam, batch, nviews, world)
        cfgd["parallelism"] += (", NCCL all-reduce of per-site gradients" if world > 1 else "") + (
            ", sdfnet sites sharded (all-gather of the SDF column)" if world > 1 and use_mlp else "")
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": elapsed_ms / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": cfgd,
            "step": ("sdfnet MLP at every site + " if use_mlp else "") +
                    "cell build + forward + backward walk" + (" + MLP backward" if use_mlp else "") +
                    (" + NCCL all-reduce" if world > 1 else ""),
            "walk": {"walk_steps_per_batch": S_mean, "mean_steps_per_ray": S_mean / batch,
                     "replayed_steps_per_batch": R_mean, "exit_record_steps": EXIT_RECORD_STEPS,
                     "visit_mean_degree": dbar,
                     "walk_order": "coherent (sorted by start site and direction)" if args.sort_rays else "as given"},
            "sdf_source": SDF_SOURCE_GPU.get(args.config, "synthetic") if use_mlp or mlp is not None else "synthetic",
            "roofline": roofline(dom, dom_bytes, dom_ms, fwd_b, bwd_b, k_fwd, k_bwd, args),
            "kernels": kernels,
            "cpu_baseline": cpu,
            "parity": parity,
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": h2d * world,
                    "d2h_bytes_per_step": d2h * world,
                    "copies": "every step: its rays, start sites and upstream gradients from pinned host memory and "
                              "its rgba back, on a copy stream that overlaps the neighbouring steps' compute; "
                              "all inside the timed region"},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clk.summary(),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_densify(args):
    """from the 1M-site medium foam, each step rebuilds the
    Delaunay adjacency on rank 0 and broadcasts it, re-sorts the per-site
    tensors, rebuilds the AABB tree and seeds 4M rays with nn on every rank,
    runs one forward + backward over this rank's share of the rays with the
    gradient all-reduce, and adds 10% new sites near the sites with the largest
    position gradient (jitter N(0, 0.005)).  Reports the per-step device time
    (max over ranks) and its phases; step 0 is untimed."""
    import torch
    import torch.distributed as dist

    import sdfoam_b200 as sdfoam
    from sdfoam_b200 import synthetic as syn
    from sdfoam_b200.densify import densify, gpu_triangulate, rebuild
    from sdfoam_b200.distributed import allreduce_grads, max_over_ranks

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime
        sys.stdout.flush()
        saved_stdout = os.dup(1)
        os.dup2(2, 1)
        try:
            dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600), device_id=dev)
            dist.barrier()
        finally:
            sys.stdout.flush()
            os.dup2(saved_stdout, 1)
            os.close(saved_stdout)
    p, sdf = syn.make_sites("medium", None, 0)
    attrs = syn.make_attributes(p, sdf, 3, "neus", seed=1)
    points = torch.from_numpy(p).to(dev)
    attributes = torch.from_numpy(attrs).to(dev)
    rays_all = np.concatenate([syn.pinhole_rays(c, tile=(8, 4)) for c in syn.views("medium")])[:4194304]
    share = (rays_all.shape[0] + world - 1) // world
    rays = torch.from_numpy(rays_all[rank * share:(rank + 1) * share]).to(dev)
    origins = rays[:, :3].contiguous()
    grad = torch.from_numpy(np.random.default_rng(7).normal(0, 1, (rays.shape[0], 4)).astype(np.float32)).to(dev)
    inv_s = torch.tensor([args.inv_s], device=dev)
    pipe = sdfoam.create_pipeline(3, "float32")
    dumped = []

    def dump_failed(pts, err):
        if args.dump_failed and not dumped:
            np.save(args.dump_failed, pts.detach().cpu().numpy())
            dumped.append(str(err))
        log(f"[densify] rebuild failed ({err}); jittering the sites and retrying")

    triangulate = gpu_triangulate(on_failure=dump_failed)
    retries = []
    gen = torch.Generator(device=dev).manual_seed(13)
    stream = torch.cuda.current_stream(dev)
    steps = max(2, args.steps)
    phases = {"rebuild_broadcast": [], "aabb_nn": [], "fwd_bwd_allreduce": [], "densify": [], "step": []}
    sites = []
    for step in range(steps):
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        ev[0].record(stream)
        perm, adj, off = rebuild(points, triangulate, world)
        retries.append(triangulate.failures)
        order = perm.long()
        points, attributes = points[order].contiguous(), attributes[order].contiguous()
        ev[1].record(stream)
        tree = sdfoam.build_aabb_tree(points)
        start = sdfoam.nn(points, tree, origins)
        ev[2].record(stream)
        fw = pipe.trace_forward(points, attributes, adj, off, rays, start, return_contribution=True,
                                alpha_mode="sdfoam", inv_s=inv_s)
        bw = pipe.trace_backward(points, attributes, adj, off, rays, start, fw["rgba"], grad, alpha_mode="sdfoam",
                                 inv_s=inv_s)
        if world > 1:
            allreduce_grads([bw["attr_grad"], bw["points_grad"]])
        ev[3].record(stream)
        sites.append(points.shape[0])
        points, attributes = densify(points, attributes, bw["points_grad"].norm(dim=1), 0.10, 0.005, gen)
        ev[4].record(stream)
        torch.cuda.synchronize()
        if step == 0:
            continue
        ms = [ev[i].elapsed_time(ev[i + 1]) for i in range(4)] + [ev[0].elapsed_time(ev[4])]
        if world > 1:
            ms = [max_over_ranks(m, dev) for m in ms]
        for k, m in zip(phases, ms):
            phases[k].append(m)
    if rank == 0:
        med = {k: float(statistics.median(v)) for k, v in phases.items()}
        line = {
            "metric": "densify + rebuild loop: ms per step (rank-0 Delaunay rebuild + broadcast, AABB + NN seeding "
                      "of 4M rays, fwd+bwd + gradient all-reduce, 10% densify)",
            "value": med["step"], "unit": "ms", "n_gpus": world, "steps": steps - 1, "warmup": 1,
            "ms_per_step": med["step"], "higher_is_better": False, "scaling": "strong", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic",
            "config": {"workload": "densify (BASELINE config 5)", "sites_first": sites[0], "sites_last": sites[-1],
                       "rays_per_step": int(rays_all.shape[0]), "parallelism": f"rays sharded over {world} GPU(s)"},
            "phases_ms": med,
            "rebuild_retries": retries,
            "sites_per_step": sites,
            "rebuild_broadcast_ms_per_step": phases["rebuild_broadcast"],
            "fwd_bwd_rays_per_s": rays_all.shape[0] / (med["fwd_bwd_allreduce"] / 1000.0),
        }
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_mlp_layer(rows: int, steps: int, warmup: int):
    """Times one tcgen05 sdfnet hidden layer (sdfoam_mlp_layer: K 264, N 256,
    softplus epilogue) on `rows` random bf16 rows; a component measurement
    for profiling, not the benchmark line."""
    import ctypes
    import torch
    from sdfoam_b200 import _lib
    lib = _lib.load()
    dev = torch.device("cuda:0")
    bf = torch.bfloat16
    g = torch.Generator(device=dev).manual_seed(0)
    x = (torch.randn((rows, 264), generator=g, device=dev) * 0.5).to(bf)
    x[:, 256] = 1
    x[:, 257:] = 0
    w = (torch.randn((256, 264), generator=g, device=dev) / 16).to(bf)
    out = torch.empty((rows, 264), dtype=bf, device=dev)
    err = torch.zeros(1, dtype=torch.int32, device=dev)
    p = lambda t: ctypes.c_void_p(t.data_ptr())
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)

    def layer():
        _lib.check(lib.sdfoam_mlp_layer(p(x), 264, 264, rows, p(w), 264, 256, None, 0, 0, 256, 1.0, p(out), 264,
                                        p(err), stream))

    for _ in range(max(warmup, 1)):
        layer()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        layer()
    e1.record()
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / steps
    gbytes = rows * 264 * 2 * 2 / 1e9
    tflop = 2 * rows * 256 * 264 / 1e12
    print(json.dumps({"component": "sdfoam_mlp_layer", "rows": rows, "ms_per_layer": ms,
                      "gb_per_s": gbytes / ms * 1e3, "tflop_per_s": tflop / ms * 1e3, "error_flag": int(err.item())}),
          flush=True)


def run_mlp_step(rows: int, steps: int, warmup: int):
    """Times the fused sdfnet forward + backward (every GEMM on the library's
    tcgen05 kernels) at `rows` random sites; a component measurement for
    profiling, not the benchmark line."""
    import torch
    dev = torch.device("cuda:0")
    pts = torch.rand((rows, 3), generator=torch.Generator().manual_seed(0)) * 2.0 - 1.0
    from sdfoam_b200 import synthetic as syn
    mlp = make_mlp(syn.Foam(pts.numpy(), None, None, None, None, 3), torch.bfloat16).to(dev)
    p = pts.to(dev).requires_grad_(True)
    g = torch.ones((rows, 1), device=dev)
    for _ in range(max(warmup, 1)):
        mlp(p).backward(g)
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(steps):
        mlp(p).backward(g)
    e1.record()
    torch.cuda.synchronize()
    from sdfoam_b200.sdfnet import check_layer_flags, mlp_flops_per_site
    check_layer_flags()
    ms = e0.elapsed_time(e1) / steps
    print(json.dumps({"component": "sdfnet fwd+bwd (fused)", "rows": rows, "ms": ms,
                      "tflop_per_s": 3 * mlp_flops_per_site(mlp) * rows / ms / 1e9}), flush=True)


def run_eikonal(rows: int, steps: int, warmup: int):
    """Times the eikonal term at `rows` points: the sdfnet's input gradient
    with its graph, the loss and its double backward, fused on the library's
    tcgen05 kernels against the same bf16 network as plain PyTorch layers
    (autograd's double backward); a component measurement, not the benchmark
    line."""
    import torch
    from sdfoam_b200 import synthetic as syn
    dev = torch.device("cuda:0")
    pts = torch.rand((rows, 3), generator=torch.Generator().manual_seed(0)) * 2.0 - 1.0
    mlp = make_mlp(syn.Foam(pts.numpy(), None, None, None, None, 3), torch.bfloat16).to(dev)
    p = pts.to(dev)
    out = {"component": "eikonal term (input gradient + loss + double backward)", "rows": rows}
    for name in ("fused", "plain_layers"):
        def step():
            x = p.clone().requires_grad_(True)
            if name == "fused":
                g = mlp.gradient(x)
            else:
                y = mlp.forward_layers(x)[:, :1]
                (g,) = torch.autograd.grad(y, x, torch.ones_like(y), create_graph=True)
            mlp.eikonal_loss(g).backward()
            for q in mlp.parameters():
                q.grad = None
        for _ in range(max(warmup, 1)):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            step()
        e1.record()
        torch.cuda.synchronize()
        out[name + "_ms"] = e0.elapsed_time(e1) / steps
    from sdfoam_b200.sdfnet import check_layer_flags
    check_layer_flags()
    print(json.dumps(out), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", default="surface", choices=sorted(CONFIGS) + ["densify"])
    ap.add_argument("--batch", type=int, default=0)
    ap.add_argument("--cpu-rays", type=int, default=1 << 20,
                    help="CPU baseline / parity sample: the first CPU_RAYS rays of the batch")
    ap.add_argument("--ref-rays", type=int, default=1 << 20,
                    help="reference arm: the first REF_RAYS rays of the batch, traced every step")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-mlp", action="store_true")
    ap.add_argument("--ray-order", default="tiles", choices=sorted(RAY_ORDERS),
                    help="tiles: view-major 8x4 pixel tiles (coherent, the headline); shuffled: training's order")
    ap.add_argument("--inv-s", type=float, default=INV_S,
                    help="NeuS sharpness (50, the headline; the model's initial exp(0.3) = 1.3499 is the other "
                         "value the survey asks for)")
    ap.add_argument("--sort-rays", action="store_true",
                    help="walk each batch in coherent order (pipeline.sort_rays), results in the caller's order")
    ap.add_argument("--dump-failed", default="", metavar="PATH",
                    help="densify: save the first site set whose rebuild failed (.npy)")
    ap.add_argument("--mlp-layer", type=int, default=0, metavar="ROWS",
                    help="time the tcgen05 MLP layer alone on ROWS rows (profiling aid)")
    ap.add_argument("--mlp-step", type=int, default=0, metavar="ROWS",
                    help="time the fused sdfnet forward + backward alone on ROWS sites (profiling aid)")
    ap.add_argument("--eikonal", type=int, default=0, metavar="ROWS",
                    help="time the eikonal term (fused vs plain layers) on ROWS points (profiling aid)")
    args = ap.parse_args()
    if args.eikonal:
        run_eikonal(args.eikonal, args.steps, args.warmup)
    elif args.mlp_layer:
        run_mlp_layer(args.mlp_layer, args.steps, args.warmup)
    elif args.mlp_step:
        run_mlp_step(args.mlp_step, args.steps, args.warmup)
    elif args.config == "densify":
        if args.impl == "ours":
            run_densify(args)
        elif int(os.environ.get("RANK", "0")) == 0:
            print(json.dumps({"impl": "reference", "unavailable": "the densify loop is a GPU-only rebuild workload; "
                              "the CPU reference arm covers the tracing configs"}), flush=True)
    elif args.impl == "reference":
        run_reference(args)
    else:
        run_gpu(args)


if __name__ == "__main__":
    main()
