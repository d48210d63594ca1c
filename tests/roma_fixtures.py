# SPDX-License-Identifier: Unlicense
"""Shared set-up of the RoMa parity tests: seeded random-init weights in
the reference's layout (written once per machine into a cache folder),
seeded synthetic tile pairs, the oracle run, and the comparison metrics
of the build's contract."""

import os
import tempfile
from pathlib import Path

import numpy as np

from coreg import synth

CACHE = Path(os.environ.get("COREG_CACHE", Path(tempfile.gettempdir()) / "coreg_cache"))


def weight_paths(seed=0):
    return synth.write_roma_weights(CACHE / "weights", seed)


_oracle_models = {}


def oracle_model(v2=True, seed=0):
    from oracle import roma_ref

    key = (v2, seed)
    if key not in _oracle_models:
        main, dino, v2p = weight_paths(seed)
        sds = [synth.read_safetensors(p) for p in (main, dino)]
        v2sd = synth.read_safetensors(v2p) if v2 else None
        _oracle_models[key] = roma_ref.Model(sds[0], sds[1], v2sd)
    return _oracle_models[key]


def tile_pair(seed, H, W):
    a, b, truth = synth.scene_pair(seed, H, W)
    return synth.tile_input(a, H, W), synth.tile_input(b, H, W), truth


def rel_l2(got, want):
    got = np.asarray(got, np.float64).reshape(-1)
    want = np.asarray(want, np.float64).reshape(-1)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-30))


def warp_px(flow_got, flow_want, H, W):
    """Per-cell distance in pixels between two normalized warps (2, H, W)."""
    dx = (np.asarray(flow_got, np.float64)[0] - flow_want[0]) * W / 2
    dy = (np.asarray(flow_got, np.float64)[1] - flow_want[1]) * H / 2
    return np.hypot(dx, dy)


def read_dump(folder, what, tile=1):
    return np.fromfile(Path(folder) / f"tile{tile:03d}_roma_{what}.f32", np.float32)
