# SPDX-License-Identifier: Unlicense
"""Benchmark of the dense-matching path: RoMa-v2ref tile pairs per second.

The unit of work is one roma_match of a tile pair at 864 x 864 with the
coarse pass at 560 (the default matcher
roma_v2ref), random init weights (seed 0) in the reference's layout,
synthetic imagery of the configuration's generator. One step is one batch
of --batch tile pairs (a slice of the configuration's 8192 x 8192 scene),
spread over the GPU's concurrent tile pipelines. Tiles are independent, so
N GPUs each process their own tiles (one process per GPU, no collective on
the data path; "scaling": "weak"): value = all tiles / max-over-ranks
device time.

Beside the headline (bfloat16, the tensor-core path) the line carries:
  fp32_mode    the same workload in float32 mode, the reference's
               arithmetic (the validation mode);
  secondary    Efficient LoFTR on 640 x 640 grey pairs and
               DISK + descriptor matching on 1024 x 1024 RGB pairs with
               2048 keypoints, through their public entry
               points, with their path-level tensor fractions.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--precision bf16|fp32]
  python bench.py --impl reference ...   (the CPU baseline arm)

Prints one JSON line (rank 0).
"""

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "i.coregistration.opencl_b200"))

H = W = 864
COARSE = 560
TILE_SRC = 1024
METRIC = "RoMa-v2ref tile pairs/s"
UNIT = "tile_pairs/s"
# Longest timed CPU work of the reference arm (whole tile pairs), seconds.
REF_BUDGET_S = 420.0
# Algorithmic FLOPs per pair of the secondary workloads (2 M N K per
# product, per image where there are two): Efficient LoFTR at 640 x 640
# (backbone 287, transformer 87, coarse matching 42, fusion 190 GFLOP) and
# DISK on two 1024 x 1024 images plus the 2048 x 2048 x 128 distance GEMM.
ELOFTR_FLOP = 605e9
# RoMa v1 at 864 with the coarse pass at 560 (about 5.25 TFLOP per pair).
ROMA_V1_FLOP = 5.25e12
DISK_FLOP = 2 * 675e9 + 2 * 2048 * 2048 * 128
CACHE = Path(os.environ.get("COREG_CACHE", "/tmp/coreg_cache"))


def dist_setup(n):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime

        import torch.distributed as dist

        # Host-side barrier and max-over-ranks of the device times only;
        # the data path has no collective.
        dist.init_process_group("gloo", timeout=datetime.timedelta(seconds=600))
    return rank, world, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist

        dist.barrier()


def allmax(world, v):
    if world == 1:
        return v
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(v)], dtype=torch.float64)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def rank_tile_seeds(rank, ntiles):
    """Seeds of the tile pairs rank processes: a contiguous block of ntiles
    per rank, disjoint across ranks (tiles are independent: no data-path
    collective)."""
    return [rank * ntiles + i for i in range(ntiles)]


def make_tiles(seeds):
    """Synthetic 1024 x 1024 tile pairs of the configuration's scene
    generator, resampled to the 864 x 864 processing size with Pillow's
    antialiased bicubic on float bands (the resampler the reference's
    prepare restates): float32 in 0..1, (3, H, W)."""
    from PIL import Image

    from coreg import synth

    out = []
    for s in seeds:
        a, b, _ = synth.scene_pair(1000 + s, TILE_SRC, TILE_SRC)
        pair = []
        for img in (a, b):
            f = img.astype(np.float32) / 255.0
            f = np.stack([np.asarray(Image.fromarray(band, mode="F").resize((W, H), Image.BICUBIC))
                          for band in f])
            pair.append(np.ascontiguousarray(np.clip(f, 0, 1), np.float32))
        out.append(pair)
    return out


class Clocks:
    """nvidia-smi samples during the timed region."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu):
        self.gpu = gpu
        self.p = None
        self.path = Path("/tmp") / f"coreg_clocks_{os.getpid()}.csv"

    def __enter__(self):
        try:
            self.f = open(self.path, "w")
            self.p = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.Q}",
                                       "--format=csv,noheader,nounits", "-lms", "100"],
                                      stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None
        time.sleep(0.3)
        return self

    def __exit__(self, *a):
        if self.p:
            self.p.terminate()
            self.p.wait()
            self.f.close()

    def summary(self):
        if not self.p or not self.path.exists():
            return None
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.path.read_text().splitlines():
            f = [x.strip() for x in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        self.path.unlink(missing_ok=True)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# ------------------------------------------------------------- work model

def work_model(Hp=H, Wp=W, Cs=COARSE, es=2):
    """Algorithmic FLOPs (tensor work) and bytes (memory-bound work) per
    tile pair of roma_v2ref, by the profiler's operation names; es is the
    element size of the refiner activations (2 in bfloat16 mode, 4 in
    float32 mode)."""
    D, c16 = 1024, Cs // 14
    n16, ntok = c16 * c16, c16 * c16 + 1
    fl, by = {}, {}

    def add(d, k, v):
        d[k] = d.get(k, 0) + v

    for N, blocks, imgs in ((ntok, 24, 2), (n16, 5, 1)):
        for name, f in (("qkv", 2 * N * D * 3 * D), ("proj", 2 * N * D * D),
                        ("fc1", 2 * N * D * 4 * D), ("fc2", 2 * N * 4 * D * D),
                        ("attention", 4 * N * N * D)):
            add(fl, name, f * blocks * imgs)
    # LayerNorm: float32 residual rows in, es-byte rows out (two per block,
    # DINOv2's final norm; both images' rows in one call).
    add(by, "layernorm", (24 * 2 + 1) * 2 * ntok * D * (4 + es) + 5 * 2 * n16 * D * (4 + es))
    add(fl, "patch_embed", 2 * 2 * n16 * 588 * D)
    add(fl, "proj16", 2 * 2 * n16 * D * 512)
    add(fl, "to_out", 2 * n16 * D * 4097)
    add(fl, "gp_gemm", 3 * 2 * n16 * n16 * 512)
    widths, blocks = (64, 128, 256, 512), (2, 2, 4, 4)

    def vgg(h, w, nblk, name):
        cin = 3
        for b in range(nblk):
            for _ in range(blocks[b]):
                add(fl, name, 2 * 2 * h * w * 9 * cin * widths[b])
                cin = widths[b]
            if b < nblk - 1:
                h, w = h // 2, w // 2

    vgg(Cs, Cs, 4, "vgg_conv3x3")
    vgg(Cs, Cs, 3, "vgg_conv3x3")
    vgg(Hp, Wp, 3, "vgg_conv3x3")
    add(fl, "vgg_proj", 2 * 2 * (Cs // 8) ** 2 * 512 * 512)
    for hh, ww in ((Cs, Cs), (Hp, Wp)):
        for sc, fin, fo in ((4, 256, 192), (2, 128, 48), (1, 64, 12)):
            add(fl, "vgg2_proj", 2 * 2 * (hh // sc) * (ww // sc) * fin * fo)

    def refiner(n, cin, feat, r, nout):
        add(fl, "refiner_out", 2 * n * cin * nout)
        if es == 2 and cin in (32, 64, 128):
            # The fused block kernel (bfloat16): the product and the
            # depthwise taps; its input read and output written once.
            add(fl, "refiner_block", 9 * (2 * n * cin * cin + 2 * 25 * n * cin))
            add(by, "refiner_block", 9 * 2 * n * cin * es)
        else:
            add(fl, "refiner_pw", 9 * 2 * n * cin * cin)
            add(fl, "roma_dwconv5", 9 * 2 * 25 * n * cin)
            add(by, "roma_dwconv5", 9 * 2 * n * cin * es)
        if r:
            add(fl, "roma_local_corr", 2 * (2 * r + 2) ** 2 * feat * n)

    refiner(c16 * c16, 1377, 512, 7, 3)
    refiner((Cs // 8) ** 2, 1137, 512, 3, 3)
    for hh, ww in ((Cs, Cs), (Hp, Wp)):
        for sc, cin, feat, r in ((4, 512, 192, 3), (2, 128, 48, 1), (1, 32, 12, 0)):
            refiner((hh // sc) * (ww // sc), cin, feat, r, 6)
    return fl, by


def profile_step(lib, dev, net, dA, dB):
    """One profiled (per-launch CUDA events, serialized) tile: {name: (ms,
    calls)}."""
    import ctypes

    lib.ops_report_reset()
    dev.ocl.profile = 1
    net.match_dev(dA, dB)
    dev.finish()
    dev.ocl.profile = 0
    n = lib.ops_report_text(None, 0)
    buf = ctypes.create_string_buffer(n)
    lib.ops_report_text(buf, n)
    out = {}
    for line in buf.value.decode().splitlines():
        name, ms, calls = line.rsplit(" ", 2)
        out[name] = (float(ms), int(calls))
    return out


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return d["hbm_gbs"], d["bf16_tflops"], "measured"
    return 6650.0, 1590.0, "fallback"


def traffic_from_profiles(kernel):
    """DRAM bytes per launch of `kernel` from the committed ncu summary, if
    one exists (profiles/roofline_traffic.json), else None."""
    p = ROOT / "profiles" / "roofline_traffic.json"
    if p.exists():
        d = json.loads(p.read_text())
        v = d.get(kernel)
        if v:
            return v.get("dram_bytes_per_launch")
    return None


# -------------------------------------------------------------- CPU arm

def cpu_sample(tiles, threads, reps=1, warmup=0, budget_s=None):
    """The oracle (the reference's roma.c restated, torch float32 on the
    host cores) on full tile pairs: seconds per timed pair, after `warmup`
    untimed pairs; stops early once `budget_s` seconds of timed pairs are
    spent (at least one pair is timed)."""
    import torch

    from oracle import roma_ref
    from coreg import synth

    torch.set_num_threads(threads)
    paths = synth.write_roma_weights(CACHE / "weights", 0)
    sds = [synth.read_safetensors(p) for p in paths]
    model = roma_ref.Model(*sds)
    r = roma_ref.Runner(model, coarse=COARSE)
    times = []
    for i in range(warmup + reps):
        a, b = tiles[i % len(tiles)]
        t = time.perf_counter()
        r.run(a, b)
        if i >= warmup:
            times.append(time.perf_counter() - t)
            if budget_s is not None and sum(times) > budget_s:
                break
    return times


def bench_config(args, world):
    """The workload keys both arms print."""
    return {"workload": "roma_v2ref tile pair: coarse 560, fine 864x864 (BASELINE configs[3])",
            "tile_px": H, "coarse_px": COARSE, "tiles_per_rank": args.tiles,
            "tiles_per_step": args.batch, "pipelines_per_gpu": max(1, args.streams),
            "parallelism": f"tiles sharded over {world} GPU(s), {max(1, args.streams)} "
                           "concurrent tile pipelines (streams) per GPU",
            "l2": "no flush: every step streams the weights and activations "
                  "(> 1 GB per tile pair) through the 126 MB L2"}


def reference_arm(args, rank, world):
    """The reference's CPU implementation of the path: the oracle port on
    all host cores (the reference's OpenCL path has no OpenCL platform to
    run on). Its step is a bounded sample of the GPU arm's step, one full
    tile pair; it runs the same warm-up and timed step counts, stopping
    early (and saying so in "steps") only past REF_BUDGET_S seconds of
    timed pairs."""
    if rank != 0:
        return
    threads = os.cpu_count() or 1
    tiles = make_tiles(range(2))
    t = cpu_sample(tiles, threads, reps=max(1, args.steps), warmup=args.warmup,
                   budget_s=REF_BUDGET_S)
    v = len(t) / sum(t)
    line = {
        "impl": "reference", "metric": METRIC, "value": v, "unit": UNIT, "n_gpus": args.gpus,
        "steps": len(t), "warmup": args.warmup, "ms_per_step": 1000 * sum(t) / len(t),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded scene generator per 1024^2 tile, resampled to 864^2; "
                "random-init weights seed 0)",
        "config": bench_config(args, world),
        "cpu_baseline": {"value": v, "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": f"{len(t)} full tile pair(s), one per step, through the "
                                   "oracle (torch float32 restatement of roma.c on all host "
                                   "cores; the reference's OpenCL path cannot run: no OpenCL "
                                   "platform on the box)"},
        "e2e": {"value": v, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# -------------------------------------------------------------- GPU arm

class Pipelines:
    """S tile pipelines on one GPU, each its own backend (stream), model and
    tile graph: tiles are independent, and a second pipeline fills the SMs
    that one tile's latency-bound stages (the Gaussian-process chain,
    launch gaps, last waves) leave idle. Device-resident tiles are copied
    into a pipeline's fixed graph inputs before each launch."""

    def __init__(self, local, prec, S, tiles, weights):
        import coreg
        from coreg.roma import Roma

        main, dino, v2 = weights
        self.S = S
        self.devs = [coreg.Device(local, precision=prec) for _ in range(S)]
        self.dev = self.devs[0]
        self.lib = self.dev.lib
        self.nets = [Roma(d, main, dino, v2, H=H, W=W, coarse=COARSE) for d in self.devs]
        self.hw3 = 3 * H * W
        self.dtiles = [(self.dev.upload(a), self.dev.upload(b)) for a, b in tiles]
        self.ins = [(d.alloc(self.hw3 * 4), d.alloc(self.hw3 * 4)) for d in self.devs]
        self.kernels = [self.nets[s].graph_build(self.ins[s][0].ptr, self.ins[s][1].ptr)
                        for s in range(S)]

    def launch(self, i):
        """Tile pair i on pipeline i % S; returns the kernels launched."""
        s = i % self.S
        a, b = self.dtiles[i % len(self.dtiles)]
        for src, dst in ((a, self.ins[s][0]), (b, self.ins[s][1])):
            self.lib.ocl_copy(self.devs[s].ocl_p, src.handle, 0, dst.handle, 0, self.hw3 * 4)
        self.nets[s].graph_launch()
        return self.kernels[s]

    def sync(self):
        for d, n_ in zip(self.devs, self.nets):
            d.finish()
            n_.sync()

    def timed(self, count):
        """Device milliseconds of `count` tile pairs, round robin over the
        pipelines, between events on the first stream (the others joined
        to it at both ends), and the kernels launched."""
        import coreg

        lib, dev = self.lib, self.dev
        lib.ocl_timer_start(dev.ocl_p)
        for s in range(1, self.S):
            lib.ocl_join(self.devs[s].ocl_p, dev.ocl_p)
        kernels = sum(self.launch(i) for i in range(count))
        for s in range(1, self.S):
            lib.ocl_join(dev.ocl_p, self.devs[s].ocl_p)
        ms = lib.ocl_timer_stop(dev.ocl_p)
        coreg.check(lib)
        self.sync()
        return ms, kernels

    def close(self):
        for n_, d in zip(self.nets, self.devs):
            n_.close()
            d.close()


def fp32_mode(local, tiles, weights, count=8, S=2):
    """Tile pairs/s of the same workload in float32 mode (float32 products,
    the reference's arithmetic), device-resident tiles, after one warm-up
    tile per pipeline."""
    import coreg

    p = Pipelines(local, coreg.OPS_FP32, S, tiles, weights)
    try:
        for i in range(S):
            p.launch(i)
        p.sync()
        ms, _ = p.timed(count)
    finally:
        p.close()
    return {"value": count / (ms / 1000.0), "unit": UNIT, "dtype": "f32", "tile_pairs": count,
            "pipelines_per_gpu": S}


def secondary(local, peak_tflops, tiles, weights, S, pairs_eloftr=16, pairs_disk=4, batches=3):
    """Configs 2, 3 and 5 through their public entry points (host images
    in, host results out), wall clock per pair after a warm-up, bfloat16
    contexts: Efficient LoFTR and DISK with their synchronous calls, RoMa v1
    through the tile queue (S pipelines), batches of 8 pairs."""
    import coreg
    from coreg import synth
    from coreg.disk import Disk, nearest
    from coreg.eloftr import Eloftr
    from coreg.roma import RomaTiles

    out = {}
    q = RomaTiles([local], S, coreg.OPS_BF16, weights[0], weights[1], None, H=H, W=W,
                  coarse=COARSE)

    def get(i, a, b):
        a[...] = tiles[i % len(tiles)][0]
        b[...] = tiles[i % len(tiles)][1]

    try:
        q.run(8, get, lambda *x: None)
        t = time.perf_counter()
        n = sum(q.run(8, get, lambda *x: None) for _ in range(batches))
        sec = (time.perf_counter() - t) / n
    finally:
        q.close()
    out["roma_v1"] = {"value": 1.0 / sec, "unit": "tile_pairs/s",
                      "workload": "RoMa v1 (roma_outdoor), batches of 8 RGB 864x864 tile pairs, "
                                  "coarse 560 (BASELINE configs[2]), through roma_tiles_run",
                      "tflops": ROMA_V1_FLOP / sec / 1e12,
                      "tensor_frac": ROMA_V1_FLOP / sec / 1e12 / peak_tflops}
    rng = np.random.default_rng(2)
    side = 640
    g0 = (synth.band_limited(rng, side, side, 3.0) / 255.0).astype(np.float32)
    g1 = np.clip(np.roll(g0, (12, -9), (0, 1)) + 0.01 * rng.standard_normal(g0.shape), 0,
                 1).astype(np.float32)
    dev = coreg.Device(local, precision=coreg.OPS_BF16)
    net = Eloftr(dev, synth.write_eloftr_weights(CACHE / "weights", 0), side, side)
    try:
        net.match(g0, g1)
        t = time.perf_counter()
        for _ in range(pairs_eloftr):
            net.match(g0, g1)
        sec = (time.perf_counter() - t) / pairs_eloftr
    finally:
        net.close()
        dev.close()
    out["eloftr"] = {"value": 1.0 / sec, "unit": "pairs/s",
                     "workload": "Efficient LoFTR, 640x640 grey pair (BASELINE configs[1])",
                     "tflops": ELOFTR_FLOP / sec / 1e12,
                     "tensor_frac": ELOFTR_FLOP / sec / 1e12 / peak_tflops}
    side, n = 1024, 2048
    pairs = []
    for k in range(2):
        a, b, _ = synth.scene_pair(40 + k, side, side)
        pairs.append((synth.tile_input(a, side, side), synth.tile_input(b, side, side)))
    dev = coreg.Device(local, precision=coreg.OPS_BF16)
    d = Disk(dev, synth.write_disk_weights(CACHE / "weights", 0), side, side, nmax=n)

    def one(pair):
        _, _, da = d.detect(pair[0], n=n)
        _, _, db = d.detect(pair[1], n=n)
        nearest(dev, da, db)

    try:
        one(pairs[0])
        t = time.perf_counter()
        for i in range(pairs_disk):
            one(pairs[i % 2])
        sec = (time.perf_counter() - t) / pairs_disk
    finally:
        d.close()
        dev.close()
    out["disk"] = {"value": 1.0 / sec, "unit": "pairs/s",
                   "workload": "DISK + descriptor matching, 1024x1024 RGB pair, 2048 keypoints "
                               "(BASELINE configs[4])",
                   "tflops": DISK_FLOP / sec / 1e12,
                   "tensor_frac": DISK_FLOP / sec / 1e12 / peak_tflops}
    return out


def gpu_arm(args, rank, world, local):
    import coreg
    from coreg import synth

    prec = coreg.OPS_BF16 if args.precision == "bf16" else coreg.OPS_FP32
    if rank == 0:
        synth.write_roma_weights(CACHE / "weights", 0)
    barrier(world)
    weights = synth.write_roma_weights(CACHE / "weights", 0)
    S = max(1, args.streams)
    B = max(1, args.batch)
    ntiles = args.tiles
    tiles = make_tiles(rank_tile_seeds(rank, ntiles))
    pipes = Pipelines(local, prec, S, tiles, weights)
    lib, dev, nets = pipes.lib, pipes.dev, pipes.nets
    hw3 = pipes.hw3
    for i in range(max(args.warmup * B, S)):
        pipes.launch(i)
    pipes.sync()
    barrier(world)
    with Clocks(local) as clk:
        ms, launches = pipes.timed(args.steps * B)
    ms_max = allmax(world, ms)
    value = world * args.steps * B / (ms_max / 1000.0)

    # Roofline of the dominant kernel, from one profiled tile.
    prof = profile_step(lib, dev, nets[0], pipes.ins[0][0].ptr, pipes.ins[0][1].ptr)
    pipes.close()

    # End to end through the library's tile queue (roma_tiles.h), the call
    # a user with a scene makes: S pipelines on this GPU, each tile's host
    # images copied into a pipeline's pinned inputs, roma_match (copies in,
    # the tile, copies out), the host results handed back in tile order;
    # wall clock over as many tile pairs as the timed region.
    from coreg.roma import RomaTiles

    q = RomaTiles([local], S, prec, *weights, H=H, W=W, coarse=COARSE)

    def get(i, a, b):
        a[...] = tiles[i % ntiles][0]
        b[...] = tiles[i % ntiles][1]

    def put(i, flow, cert, sd):
        pass

    try:
        q.run(S, get, put)
        barrier(world)
        t0 = time.perf_counter()
        e2e_tiles = q.run(args.steps * B, get, put)
        e2e_ms = (time.perf_counter() - t0) * 1000.0
    finally:
        q.close()
    e2e_max = allmax(world, e2e_ms)
    e2e_value = world * e2e_tiles / (e2e_max / 1000.0)

    fl, by = work_model(es=2 if prec else 4)
    hbm, bf16, peak_kind = peaks()
    # The dominant profiled operation that has a work model and a DRAM
    # traffic figure from the committed ncu capture (operations whose
    # kernels ncu can tell apart by name), else the dominant one with a
    # work model.
    modeled = [k for k in prof if k in fl or k in by]
    traced = [k for k in modeled if traffic_from_profiles(k)]
    dom = max(traced or modeled, key=lambda k: prof[k][0])
    roof = None
    if dom in fl and (dom not in by or fl[dom] / max(by[dom], 1) > 50):
        ms_d, calls = prof[dom]
        ach = fl[dom] / (ms_d / 1000.0) / 1e12
        roof = {"bound": "tensor", "kernel": dom, "achieved": ach, "peak": bf16, "unit": "TFLOP/s",
                "frac": ach / bf16, "peak_kind": peak_kind,
                "traffic": traffic_from_profiles(dom), "launches_per_step": calls * B,
                "algorithmic_per_launch": fl[dom] / calls}
    elif dom in by:
        ms_d, calls = prof[dom]
        ach = by[dom] / (ms_d / 1000.0) / 1e9
        roof = {"bound": "hbm", "kernel": dom, "achieved": ach, "peak": hbm, "unit": "GB/s",
                "frac": ach / hbm, "peak_kind": peak_kind,
                "traffic": traffic_from_profiles(dom), "launches_per_step": calls * B,
                "algorithmic_per_launch": by[dom] / calls}
    tot_ms = sum(v[0] for v in prof.values())
    shares = sorted(((k, v[0] / tot_ms) for k, v in prof.items()), key=lambda x: -x[1])[:14]
    flops_pair = sum(fl.values())

    extra = {}
    if rank == 0 and world == 1 and not args.no_extra:
        if prec == coreg.OPS_BF16:
            extra["fp32_mode"] = fp32_mode(local, tiles, weights)
        extra["secondary"] = secondary(local, bf16, tiles, weights, S)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        threads = os.cpu_count() or 1
        t = cpu_sample(tiles, threads, reps=1)
        cpu = {"value": 1.0 / t[0], "unit": UNIT, "cores": threads, "kind": "port",
               "sample": "1 full tile pair (coarse 560, fine 864) through the oracle, torch "
                         "float32 on the host cores (the reference's OpenCL path cannot run: "
                         "no OpenCL platform on the box)"}
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_max / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "bf16" if prec else "f32",
            "data": "synthetic (seeded scene generator per 1024^2 tile, resampled to 864^2; "
                    "random-init weights seed 0)",
            "config": bench_config(args, world),
            "e2e": {"value": e2e_value, "unit": UNIT, "h2d_bytes_per_step": B * 2 * hw3 * 4,
                    "d2h_bytes_per_step": B * 4 * H * W * 4,
                    "api": "roma_tiles_run (host images into pinned inputs, roma_match per "
                           "tile, host results in tile order)"},
            "gpu_launches": launches,
            "roofline": roof,
            "path_tflops": flops_pair / (ms_max / (args.steps * B) / 1000.0) / 1e12,
            "time_shares": {k: round(v, 4) for k, v in shares},
            "profiled_tile_ms": round(tot_ms, 3),
            "cpu_baseline": cpu,
            "clocks": clk.summary(),
        }
        line.update(extra)
        print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--precision", default="bf16", choices=["bf16", "fp32"])
    ap.add_argument("--tiles", type=int, default=4, help="distinct tile pairs per GPU")
    ap.add_argument("--batch", type=int, default=8, help="tile pairs per step")
    ap.add_argument("--no-cpu", action="store_true", help="skip the CPU baseline sample")
    ap.add_argument("--no-extra", action="store_true",
                    help="skip the float32-mode and secondary workloads")
    ap.add_argument("--streams", type=int, default=4,
                    help="concurrent tile pipelines (streams, models) per GPU")
    args = ap.parse_args()
    rank, world, local = dist_setup(args.gpus)
    if args.impl == "reference":
        reference_arm(args, rank, world)
    else:
        gpu_arm(args, rank, world, local)
    if world > 1:
        import torch.distributed as dist

        barrier(world)
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
