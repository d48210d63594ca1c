# SPDX-License-Identifier: Unlicense
"""RoMa parity: the CUDA device stage (roma_match through the C-ABI)
against the oracle (oracle/roma_ref.py, the reference's roma.c restated),
stage by stage through the reference's own dump points (roma.c:1188-1227)
and on the final warp, certainty and standard deviation (GPU).

Contract (float32 mode): intermediate tensors within a relative L2 error
of 1e-5 per operation (checked per stage with the bound the stage's depth
allows, below), dense warp within 0.05 px mean and 0.25 px p99, certainty
within 1e-2 absolute. bfloat16 mode: per-stage relative L2 within 2e-2.
Sizes: coarse pass 224 (16 x 16 DINOv2 tokens) and 128 x 128 tiles, so that
the oracle finishes in seconds; the benchmarked 560 / 864 size is checked
in tests/test_roma_headline_gpu.py.
"""

import numpy as np
import pytest

import coreg
from coreg.roma import Roma
from roma_fixtures import oracle_model, read_dump, rel_l2, tile_pair, warp_px, weight_paths

# Relative L2 bounds per dump point in float32 mode: 1e-5 per operation,
# times the depth of the chain that produced it (24 ViT blocks for the
# DINOv2 features, the GP solve's conditioning on top).
FP32_STAGE = {"in_c_0": 1e-6, "in_c_1": 1e-6, "in_f_0": 1e-6, "in_f_1": 1e-6,
              "dino_0": 1e-5, "dino_1": 1e-5, "gp": 5e-4, "cls_flow": 1e-5,
              "p0_s8_flow": 1e-5}


def run_pair(dev, tmp_path, v2, H, W, coarse, seed=1):
    main, dino, v2p = weight_paths()
    A, B, _ = tile_pair(seed, H, W)
    net = Roma(dev, main, dino, v2p if v2 else None, H=H, W=W, coarse=coarse)
    try:
        flow, cert, sd = net.match(A, B, dump=tmp_path)
    finally:
        net.close()
    from oracle import roma_ref

    r = roma_ref.Runner(oracle_model(v2), coarse=coarse)
    res = r.run(A, B)
    return (flow, cert, sd), res, r.dumps


def check_final(got, want, H, W, px_mean=0.05, px_p99=0.25, cert_abs=1e-2):
    flow, cert, sd = got
    d = warp_px(flow, want[0], H, W)
    report = dict(px_mean=float(d.mean()), px_p99=float(np.percentile(d, 99)),
                  cert_max=float(np.abs(cert - want[1]).max()))
    assert report["px_mean"] <= px_mean, report
    assert report["px_p99"] <= px_p99, report
    assert report["cert_max"] <= cert_abs, report
    if sd is not None:
        ok = np.isfinite(want[2]) & np.isfinite(sd)
        assert (np.isfinite(sd) == np.isfinite(want[2])).mean() > 0.999
        assert rel_l2(sd[ok], want[2][ok]) <= 1e-2
    return report


@pytest.mark.gpu
@pytest.mark.parametrize("v2", [True, False], ids=["roma_v2ref", "roma"])
def test_roma_fp32_parity(tmp_path, v2):
    dev = coreg.Device(0, precision=coreg.OPS_FP32)
    H = W = 128
    got, want, dumps = run_pair(dev, tmp_path, v2, H, W, coarse=224)
    for name, bound in FP32_STAGE.items():
        g = read_dump(tmp_path, name)
        assert rel_l2(g, dumps[name].numpy()) <= bound, (name, rel_l2(g, dumps[name].numpy()))
    check_final(got, want, H, W)
    dev.close()


@pytest.mark.gpu
def test_roma_bf16_stages(tmp_path):
    """bfloat16 tensor-core mode: every dumped stage within 2e-2 relative
    L2 of the float32 oracle up to the GP; the warp reported."""
    dev = coreg.Device(0, precision=coreg.OPS_BF16)
    H = W = 128
    got, want, dumps = run_pair(dev, tmp_path, True, H, W, coarse=224)
    for name in ("in_c_0", "in_c_1", "dino_0", "dino_1"):
        g = read_dump(tmp_path, name)
        assert rel_l2(g, dumps[name].numpy()) <= 2e-2, (name, rel_l2(g, dumps[name].numpy()))
    flow = got[0]
    assert np.isfinite(flow).all() and np.abs(flow).max() <= 1.0
    dev.close()


@pytest.mark.gpu
def test_two_concurrent_pipelines_match_solo_runs():
    """Two models on one device, each with its own backend (stream), run
    roma_match at the same time from two host threads (the way bench.py
    fills a GPU): each result equals the same model's solo result
    bit for bit."""
    import threading

    H = W = 128
    main, dino, v2p = weight_paths()
    devs = [coreg.Device(0, precision=coreg.OPS_BF16) for _ in range(2)]
    nets = [Roma(d, main, dino, v2p, H=H, W=W, coarse=224) for d in devs]
    try:
        pairs = [tile_pair(s, H, W)[:2] for s in (3, 4)]
        solo = [tuple(np.copy(x) for x in nets[k].match(*pairs[k])) for k in range(2)]
        out = [None, None]
        errs = []

        def run(k):
            try:
                out[k] = tuple(np.copy(x) for x in nets[k].match(*pairs[k]))
            except Exception as e:
                errs.append(e)

        th = [threading.Thread(target=run, args=(k,)) for k in range(2)]
        for t in th:
            t.start()
        for t in th:
            t.join()
        assert not errs, errs
        for k in range(2):
            for a, b in zip(out[k], solo[k]):
                assert np.array_equal(a, b, equal_nan=True)
    finally:
        for n_, d in zip(nets, devs):
            n_.close()
            d.close()
