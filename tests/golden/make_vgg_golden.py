# SPDX-License-Identifier: Unlicense
"""Generate tests/golden/vgg_golden.npz: RoMa's VGG19-BN feature pyramid
(torchvision's vgg19_bn features, which RoMa's CNN encoder is, in eval mode)
evaluated by torchvision in float64 with the seeded synthetic weights of
coreg.synth.roma_weights(0) (encoder.cnn.layers.<index> in torchvision's
feature indexing), on a seeded 3 x 32 x 32 input. Stores as float32 the
input and the activations that end each of the four blocks (after the
ReLU of the block's last convolution, before its pooling):

    img, f1 (64, 32, 32), f2 (128, 16, 16), f4 (256, 8, 8), f8 (512, 4, 4)

Needs torchvision and torch (present in the build container); run from the
repository root:

    python tests/golden/make_vgg_golden.py
"""

import sys
from pathlib import Path

import numpy as np
import torch
import torchvision

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT / "i.coregistration.opencl_b200"))

from coreg import synth  # noqa: E402

ENDS = {5: "f1", 12: "f2", 25: "f4", 38: "f8"}  # ReLU after each block's last convolution


def main():
    main_sd = synth.roma_weights(0)[0]
    pre = "encoder.cnn.layers."
    feats = torchvision.models.vgg19_bn(weights=None).features[:40].double().eval()
    state = {k[len(pre):]: torch.from_numpy(np.asarray(v, np.float64))
             for k, v in main_sd.items() if k.startswith(pre)}
    res = feats.load_state_dict(state, strict=False)
    missing = [k for k in res.missing_keys if not k.endswith("num_batches_tracked")]
    if res.unexpected_keys or missing:
        raise SystemExit(f"weight names differ: {missing[:5]} {res.unexpected_keys[:5]}")
    img = np.random.default_rng(11).standard_normal((3, 32, 32)).astype(np.float32)
    out = {"img": img}
    x = torch.from_numpy(img).double()[None]
    with torch.no_grad():
        for i, layer in enumerate(feats):
            x = layer(x)
            if i in ENDS:
                out[ENDS[i]] = x[0].numpy().astype(np.float32)
    dst = ROOT / "tests" / "golden" / "vgg_golden.npz"
    np.savez_compressed(dst, **out)
    print(f"{dst} ({dst.stat().st_size} bytes)")


if __name__ == "__main__":
    main()
