# SPDX-License-Identifier: Unlicense
"""The measurement's bookkeeping (CPU): bench.py's algorithmic work model
against the survey's derived figure for roma_v2ref at coarse 560 / fine
864 (about 4.78 TFLOP per tile pair: the ViT about half, the VGG
encoders about 30 %), and the committed ncu traffic file that bench.py's
roofline reads: every category in it has a work-model entry, a positive
launch count and DRAM bytes per launch."""

import json
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parents[1]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

import bench  # noqa: E402


def test_work_model_matches_the_derived_figure():
    fl, by = bench.work_model()
    total = sum(fl.values())
    assert abs(total / 4.78e12 - 1) < 0.01, total
    vit = sum(fl[k] for k in ("qkv", "proj", "fc1", "fc2", "attention"))
    # The ViT blocks of DINOv2 (both images) and of the coordinate decoder.
    assert 0.50 < vit / total < 0.58, vit / total
    assert 0.27 < fl["vgg_conv3x3"] / total < 0.33, fl["vgg_conv3x3"] / total
    # bfloat16 refiner activations (2 bytes) against float32 (4): twice the bytes.
    fl32, by32 = bench.work_model(es=4)
    assert by32["roma_dwconv5"] > 0 and "refiner_block" not in by32
    assert by["refiner_block"] > 0


def test_roofline_traffic_file_covers_modelled_categories():
    d = json.loads((ROOT / "profiles" / "roofline_traffic.json").read_text())
    fl, by = bench.work_model()
    cats = {k: v for k, v in d.items() if not k.startswith("_")}
    assert "vgg_conv3x3" in cats
    for name, v in cats.items():
        assert name in fl or name in by, name
        assert v["launches"] > 0 and v["dram_bytes_per_launch"] > 0, (name, v)
        assert bench.traffic_from_profiles(name) == v["dram_bytes_per_launch"]
