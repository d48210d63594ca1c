# SPDX-License-Identifier: Unlicense
"""Generate tests/golden/roma_ref_golden.npz from the reference's own RoMa.

Runs the reference's roma_load (+ roma_load_v2), roma_alloc and roma_match
(roma.c:398-544, 559-643, 1357-1435), unchanged, over its ops.c and OpenCL
kernels on the CPU (oracle/_ref/libref_cpu.so, built by oracle/Makefile
from the reference checkout; the OpenCL runtime is oracle/cl_backend_emul.c)
with the seeded random-init weights of the tests (coreg.synth, seed 0) on the
seeded tile pair of the RoMa GPU tests (seed 1, 128 x 128). The coarse pass
runs at the reference's fixed 560 px, so each model takes about an hour on
one core; roma_v2ref and roma (v1) run in two processes side by side.

The reference writes its own debug dumps (roma.c:1188-1227); the fixture
keeps them, thinned where they are large:
  dino_0 / dino_1   every 32nd token, all 1024 channels ((1024, 50) each);
  gp                every 16th token ((100, 512));
  cls_flow, cls_cert, and every refiner's warp and certainty (confidence
  for RoMa v2) up to 140 x 140 cells whole, larger grids every 4th (280)
  or 8th (560) cell in each axis;
  flow, cert (and sd for v2) at the tile size, whole.
Keys are prefixed with the model ("v2_" or "v1_"); "tile_seed", "H", "W" and
"coarse" record the inputs. Run from the repository root:

    python tests/golden/make_roma_ref_golden.py
"""

import ctypes as C
import multiprocessing as mp
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
for p in (ROOT, ROOT / "i.coregistration.opencl_b200", ROOT / "tests"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))

LIB = ROOT / "oracle" / "_ref" / "libref_cpu.so"
OUT = Path(__file__).resolve().parent / "roma_ref_golden.npz"
H = W = 128
TILE_SEED = 1
COARSE = 560
C16 = COARSE // 14
N16 = C16 * C16


def run_model(v2, folder):
    """The reference's roma_match of the fixture's tile pair, dumps into
    folder; returns the seconds it took."""
    from roma_fixtures import tile_pair, weight_paths

    main, dino, v2p = weight_paths()
    A, B, _ = tile_pair(TILE_SEED, H, W)
    lib = C.CDLL(str(LIB))
    P, I = C.c_void_p, C.c_int
    lib.ref_roma_match.restype = None
    lib.ref_roma_match.argtypes = [C.c_char_p, C.c_char_p, C.c_char_p, I, I, P, P, C.c_char_p,
                                   P, P, P]
    flow = np.zeros((2, H, W), np.float32)
    cert = np.zeros((H, W), np.float32)
    sd = np.zeros((H, W), np.float32)
    A = np.ascontiguousarray(A, np.float32)
    B = np.ascontiguousarray(B, np.float32)
    t = time.time()
    lib.ref_roma_match(str(main).encode(), str(dino).encode(),
                       str(v2p).encode() if v2 else None, H, W, A.ctypes.data, B.ctypes.data,
                       str(folder).encode(), flow.ctypes.data, cert.ctypes.data,
                       sd.ctypes.data)
    return time.time() - t


def read(folder, what):
    return np.fromfile(Path(folder) / f"tile001_roma_{what}.f32", np.float32)


def thin(v, channels, side):
    """A (channels, side * side) grid dump, every 4th (side 280) or 8th
    (side 560) cell in each axis; smaller grids whole."""
    g = v.reshape(channels, side, side)
    step = 1 if side <= 140 else (4 if side <= 280 else 8)
    return np.ascontiguousarray(g[:, ::step, ::step])


def scales(v2):
    """(pass, dump name, grid side, certainty channels) of every refiner
    dump roma_match writes (roma.c:1232-1306)."""
    out = [(0, "s16", C16, 1), (0, "s8", COARSE // 8, 1)]
    if v2:
        for p, side in ((0, COARSE), (1, H)):
            out += [(p, f"v2s{s}", side // s, 4) for s in (4, 2, 1)]
    else:
        out += [(0, f"s{s}", COARSE // s, 1) for s in (4, 2, 1)]
        out += [(1, f"s{s}", H // s, 1) for s in (8, 4, 2, 1)]
    return out


def collect(folder, v2, prefix):
    out = {}
    for k in (0, 1):
        out[f"{prefix}dino_{k}"] = read(folder, f"dino_{k}").reshape(1024, N16)[:, ::32].copy()
    out[prefix + "gp"] = read(folder, "gp").reshape(N16, 512)[::16].copy()
    out[prefix + "cls_flow"] = read(folder, "cls_flow").reshape(2, N16)
    out[prefix + "cls_cert"] = read(folder, "cls_cert")
    for p, name, side, cc in scales(v2):
        out[f"{prefix}p{p}_{name}_flow"] = thin(read(folder, f"p{p}_{name}_flow"), 2, side)
        what = "conf" if cc == 4 else "cert"
        out[f"{prefix}p{p}_{name}_{what}"] = thin(read(folder, f"p{p}_{name}_{what}"), cc, side)
    out[prefix + "flow"] = read(folder, "flow").reshape(2, H, W)
    out[prefix + "cert"] = read(folder, "cert").reshape(H, W)
    if v2:
        out[prefix + "sd"] = read(folder, "sd").reshape(H, W)
    return out


def job(v2, folder, q):
    q.put((v2, run_model(v2, folder)))


def main():
    if not LIB.exists():
        sys.exit("oracle/_ref/libref_cpu.so is missing: make -C oracle REF=<reference checkout>")
    # Weights are written before the workers start.
    from roma_fixtures import weight_paths

    weight_paths()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with tempfile.TemporaryDirectory() as d2, tempfile.TemporaryDirectory() as d1:
        procs = [ctx.Process(target=job, args=(v2, d, q)) for v2, d in ((True, d2), (False, d1))]
        for p in procs:
            p.start()
        secs = dict(q.get() for _ in procs)
        for p in procs:
            p.join()
            if p.exitcode:
                sys.exit(f"reference run failed ({p.exitcode})")
        out = {"tile_seed": np.int64(TILE_SEED), "H": np.int64(H), "W": np.int64(W),
               "coarse": np.int64(COARSE)}
        out.update(collect(d2, True, "v2_"))
        out.update(collect(d1, False, "v1_"))
    np.savez_compressed(OUT, **out)
    print(f"wrote {OUT} ({OUT.stat().st_size} bytes); reference seconds: "
          f"v2 {secs[True]:.0f}, v1 {secs[False]:.0f}")


if __name__ == "__main__":
    main()
