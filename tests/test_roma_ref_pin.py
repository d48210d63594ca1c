# SPDX-License-Identifier: Unlicense
"""RoMa's whole tile pinned to the reference itself: the reference's own
roma_load / roma_load_v2 / roma_alloc / roma_match (roma.c:398-1435), run
unchanged on the CPU over the OpenCL emulation, wrote its debug dumps
(roma.c:1188-1227) for the seeded weights and tile pair of the RoMa tests
(128 x 128 tile, the reference's fixed 560 px coarse pass; both roma_v2ref
and roma v1). tests/golden/make_roma_ref_golden.py made the fixture
tests/golden/roma_ref_golden.npz from them.

CPU: the oracle (oracle/roma_ref.py) against the fixture, stage by stage:
the DINOv2 features and the GP posterior (sampled tokens), the decoder's
coarse warp and certainty (decoder blocks, to_out and cls_to_flow), every
refiner's warp and certainty of both passes (RoMa v1's five refiners, the
v2 refiners), and the final warp, certainty and sd. This pins the wiring
of the coarse pass that the piecewise pins leave open.

GPU: the device stage in float32 mode (roma_match through the C-ABI)
against the same fixture, with the same bounds. The decoder's 4096-way
anchor choice (first-index argmax, roma_kernels.cl:46-102) is a hard
decision: on this smooth, upsampled tile some tokens' two best anchor
logits lie closer than float32 rounding in another summation order moves
them. The oracle (which keeps the reference's anchors here, see the CPU
test) gives every token's margin; a token may take another anchor only
where its margin is below twice the device's largest logit error, and at
most 1 % of the tokens do. At the other tokens the coarse warp must match
the fixture; downstream of the anchors the device stages are compared
with the oracle run from the device's own anchors (forced), under the same
float32 bounds, and the final warp, certainty and sd with that run's.

Bounds (the build's float32 contract): relative L2 1e-5 per warp stage, 5e-4
for the GP posterior (the kernel matrices are float32, summed in another
order) and for the certainty logits downstream of it; warp within 0.05 px
mean and 0.25 px p99, certainty within 1e-2. Measured for the oracle: warps
within 2.2e-6, the GP 3.9e-4, certainties within 8.5e-5, the final warp
0.0000 px mean and 0.0003 px p99, the final certainty within 4.2e-5."""

from pathlib import Path

import numpy as np
import pytest

from roma_fixtures import oracle_model, read_dump, rel_l2, tile_pair, warp_px, weight_paths

GOLDEN = Path(__file__).resolve().parent / "golden" / "roma_ref_golden.npz"
COARSE = 560


@pytest.fixture(scope="module")
def golden():
    if not GOLDEN.exists():
        pytest.skip("tests/golden/roma_ref_golden.npz not generated")
    return dict(np.load(GOLDEN))


def thin_like(v, want):
    """A full (C, side * side) dump thinned the way the fixture stores it."""
    C, h, w = want.shape
    side = int(round(np.sqrt(np.asarray(v).size // C)))
    g = np.asarray(v, np.float64).reshape(C, side, side)
    step = side // h if side != h else 1
    return g[:, ::step, ::step]


def stage_bound(name):
    # The GP posterior carries the float32 rounding of its kernel matrices
    # (summed in a different order than the reference's), and the
    # certainty logits downstream of it carry the same; the warps stay
    # within the float32 bound.
    return 5e-4 if name.endswith(("gp", "cert", "conf")) else 1e-5


def compare(g, dumps, prefix, H, W, final):
    """Every stage of the fixture against dumps (name -> array), then the
    final results (flow, cert, sd or None; final None: stages only)."""
    n16 = (COARSE // 14) ** 2
    for key, want in g.items():
        if not key.startswith(prefix) or key[len(prefix):] in ("flow", "cert", "sd"):
            continue
        name = key[len(prefix):]
        got = np.asarray(dumps[name], np.float64)
        if name.startswith("dino_"):
            got = got.reshape(1024, n16)[:, ::32]
        elif name == "gp":
            got = got.reshape(n16, 512)[::16]
        elif name.startswith("p"):
            got = thin_like(got, want)
        e = rel_l2(got, want)
        assert e <= stage_bound(name), (prefix, name, e)
    if final is None:
        return
    flow, cert, sd = final
    d = warp_px(flow, g[prefix + "flow"], H, W)
    assert d.mean() <= 0.05 and np.percentile(d, 99) <= 0.25, (prefix, d.mean())
    assert np.abs(cert - g[prefix + "cert"]).max() <= 1e-2
    if sd is not None:
        want = g[prefix + "sd"]
        ok = np.isfinite(want) & np.isfinite(sd)
        assert (np.isfinite(sd) == np.isfinite(want)).mean() > 0.999
        assert rel_l2(sd[ok], want[ok]) <= 1e-2


@pytest.mark.slow
@pytest.mark.parametrize("v2", [True, False], ids=["roma_v2ref", "roma"])
def test_oracle_matches_the_reference_roma_match(golden, v2):
    from oracle import roma_ref

    H, W = int(golden["H"]), int(golden["W"])
    assert int(golden["coarse"]) == COARSE
    A, B, _ = tile_pair(int(golden["tile_seed"]), H, W)
    r = roma_ref.Runner(oracle_model(v2), coarse=COARSE)
    res = r.run(A, B)
    dumps = {k: v.numpy() for k, v in r.dumps.items()}
    compare(golden, dumps, "v2_" if v2 else "v1_", H, W, res if v2 else (res[0], res[1], None))


NCLS = 4096
# Stages upstream of the anchor choice, checked against the fixture itself.
UPSTREAM = ("dino_0", "dino_1", "gp")


@pytest.mark.gpu
@pytest.mark.parametrize("v2", [True, False], ids=["roma_v2ref", "roma"])
def test_gpu_fp32_matches_the_reference_roma_match(tmp_path, golden, v2):
    import coreg
    from coreg.roma import Roma
    from oracle import roma_ref

    H, W = int(golden["H"]), int(golden["W"])
    A, B, _ = tile_pair(int(golden["tile_seed"]), H, W)
    main, dino, v2p = weight_paths()
    dev = coreg.Device(0, precision=coreg.OPS_FP32)
    try:
        net = Roma(dev, main, dino, v2p if v2 else None, H=H, W=W, coarse=COARSE)
        try:
            flow, cert, sd = net.match(A, B, dump=tmp_path)
        finally:
            net.close()
    finally:
        dev.close()
    prefix = "v2_" if v2 else "v1_"
    n16 = (COARSE // 14) ** 2
    names = [k[len(prefix):] for k in golden if k.startswith(prefix)]
    dumps = {n: read_dump(tmp_path, n) for n in names if n not in ("flow", "cert", "sd")}
    # Upstream of the anchors: the fixture itself.
    compare({prefix + k: golden[prefix + k] for k in UPSTREAM}, dumps, prefix, H, W, None)

    # The anchors against the oracle's (the reference's, on this tile).
    r = roma_ref.Runner(oracle_model(v2), coarse=COARSE)
    r.run(A, B)
    Lr = r.dumps["cls_logits"].numpy().astype(np.float64)
    Lg = read_dump(tmp_path, "cls_logits").reshape(n16, NCLS + 1).astype(np.float64)
    err = np.abs(Lg - Lr).max()
    top2 = np.sort(Lr[:, :NCLS], axis=1)[:, -2:]
    margin = top2[:, 1] - top2[:, 0]
    mode_g = np.argmax(Lg[:, :NCLS], axis=1)
    flipped = mode_g != np.argmax(Lr[:, :NCLS], axis=1)
    print(prefix, "anchors taken otherwise:", int(flipped.sum()), "logit error", err,
          "their margins", margin[flipped])
    assert not (flipped & (margin > 2 * err)).any(), (err, margin[flipped])
    assert flipped.mean() <= 0.01, flipped.mean()
    # The coarse warp at the tokens that keep their anchor: the fixture's.
    cf = dumps["cls_flow"].reshape(2, n16)[:, ~flipped]
    e = rel_l2(cf, golden[prefix + "cls_flow"][:, ~flipped])
    assert e <= 1e-5, ("cls_flow", e)

    # Downstream: the oracle from the device's anchors.
    rf = roma_ref.Runner(oracle_model(v2), coarse=COARSE)
    rf.force_mode = mode_g
    res = rf.run(A, B)
    forced = {prefix + k: thin_like(v.numpy(), golden[prefix + k]) if k.startswith("p") else
              v.numpy() for k, v in rf.dumps.items() if prefix + k in golden and
              k not in UPSTREAM}
    forced[prefix + "flow"] = res[0]
    forced[prefix + "cert"] = res[1]
    if v2:
        forced[prefix + "sd"] = res[2]
    compare(forced, dumps, prefix, H, W, (flow, cert, sd if v2 else None))
