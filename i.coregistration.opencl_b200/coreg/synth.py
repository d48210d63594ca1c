# SPDX-License-Identifier: Unlicense
"""Seeded synthetic data of the benchmarks and tests: random-init weights
in the reference's tensor names and shapes (the state_dicts that
roma_load / roma_load_v2 read, roma.c:217-531), written as safetensors,
and synthetic imagery with the value distributions of the benchmark
configurations. No pretrained weights or datasets are involved.
"""

import json
import math
from pathlib import Path

import numpy as np

VIT_DIM, VIT_DEPTH, DEC_DEPTH, MLP = 1024, 24, 5, 4
REF_SCALE = (16, 8, 4, 2, 1)
REF_FEAT = (512, 512, 256, 64, 9)
REF_EMB = (128, 64, 32, 16, 6)
REF_RADIUS = (7, 3, 2, 0, 0)
PROJ_IN = (1024, 512, 256, 128, 64)
REF2_SCALE = (4, 2, 1)
REF2_IN = (256, 128, 64)
REF2_FEAT = (192, 48, 12)
REF2_EMB = (79, 23, 8)
REF2_RADIUS = (3, 1, 0)
VGG_BLOCKS = (2, 2, 4, 4)
VGG_WIDTH = (64, 128, 256, 512)


def write_safetensors(path, tensors):
    """Write {name: float32 array} as a safetensors file."""
    header, off = {}, 0
    order = list(tensors)
    for k in order:
        a = np.ascontiguousarray(tensors[k], np.float32)
        tensors[k] = a
        header[k] = {"dtype": "F32", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    h = json.dumps(header, separators=(",", ":")).encode()
    h += b" " * ((8 - len(h) % 8) % 8)
    with open(path, "wb") as f:
        f.write(len(h).to_bytes(8, "little"))
        f.write(h)
        for k in order:
            f.write(tensors[k].tobytes())


def read_safetensors(path):
    """{name: float32 array} of a safetensors file (F32 / F16 / BF16)."""
    data = Path(path).read_bytes()
    n = int.from_bytes(data[:8], "little")
    header = json.loads(data[8:8 + n])
    out = {}
    base = 8 + n
    for k, v in header.items():
        if k == "__metadata__":
            continue
        a, b = v["data_offsets"]
        raw = data[base + a: base + b]
        if v["dtype"] == "F32":
            arr = np.frombuffer(raw, np.float32)
        elif v["dtype"] == "F16":
            arr = np.frombuffer(raw, np.float16).astype(np.float32)
        elif v["dtype"] == "BF16":
            arr = (np.frombuffer(raw, np.uint16).astype(np.uint32) << 16).view(np.float32)
        else:
            continue
        out[k] = arr.reshape(v["shape"]).copy()
    return out


class Gen:
    def __init__(self, seed):
        self.rng = np.random.default_rng(seed)

    def normal(self, shape, std):
        return (self.rng.standard_normal(shape, dtype=np.float32) * np.float32(std)).astype(np.float32)

    def uniform(self, shape, lo, hi):
        return self.rng.uniform(lo, hi, shape).astype(np.float32)


def _bn(g, d, name, c):
    d[f"{name}.weight"] = g.uniform((c,), 0.8, 1.2)
    d[f"{name}.bias"] = g.normal((c,), 0.1)
    d[f"{name}.running_mean"] = g.normal((c,), 0.1)
    d[f"{name}.running_var"] = g.uniform((c,), 0.8, 1.5)


def _vgg(g, d, pre, nblk):
    idx, cin = 0, 3
    for blk in range(nblk):
        for _ in range(VGG_BLOCKS[blk]):
            co = VGG_WIDTH[blk]
            d[f"{pre}.{idx}.weight"] = g.normal((co, cin, 3, 3), math.sqrt(2.0 / (9 * cin)))
            d[f"{pre}.{idx}.bias"] = g.normal((co,), 0.05)
            _bn(g, d, f"{pre}.{idx + 1}", co)
            cin = co
            idx += 3
        idx += 1


def _block(g, d, pre, D, qkv_bias, ls):
    d[f"{pre}.norm1.weight"] = 1.0 + g.normal((D,), 0.02)
    d[f"{pre}.norm1.bias"] = g.normal((D,), 0.02)
    d[f"{pre}.attn.qkv.weight"] = g.normal((3 * D, D), 0.02)
    if qkv_bias:
        d[f"{pre}.attn.qkv.bias"] = g.normal((3 * D,), 0.02)
    d[f"{pre}.attn.proj.weight"] = g.normal((D, D), 0.02)
    d[f"{pre}.attn.proj.bias"] = g.normal((D,), 0.02)
    d[f"{pre}.norm2.weight"] = 1.0 + g.normal((D,), 0.02)
    d[f"{pre}.norm2.bias"] = g.normal((D,), 0.02)
    d[f"{pre}.mlp.fc1.weight"] = g.normal((MLP * D, D), 0.02)
    d[f"{pre}.mlp.fc1.bias"] = g.normal((MLP * D,), 0.02)
    d[f"{pre}.mlp.fc2.weight"] = g.normal((D, MLP * D), 0.02)
    d[f"{pre}.mlp.fc2.bias"] = g.normal((D,), 0.02)
    if ls is not None:
        d[f"{pre}.ls1.gamma"] = np.full((D,), ls, np.float32) if np.isscalar(ls) else ls
        d[f"{pre}.ls2.gamma"] = np.full((D,), ls, np.float32) if np.isscalar(ls) else ls


def _ref_blocks(g, d, pre, cin, v2):
    for b in range(9):
        blk = f"{pre}.block1" if b == 0 else f"{pre}.hidden_blocks.{b - 1}"
        dw, bn, pw = ((f"{blk}.conv_depthwise", f"{blk}.norm", f"{blk}.conv_pointwise") if v2
                      else (f"{blk}.0", f"{blk}.1", f"{blk}.3"))
        d[f"{dw}.weight"] = g.normal((cin, 1, 5, 5), math.sqrt(2.0 / 25))
        d[f"{dw}.bias"] = g.normal((cin,), 0.05)
        _bn(g, d, bn, cin)
        d[f"{pw}.weight"] = g.normal((cin, cin, 1, 1), math.sqrt(1.0 / cin))
        d[f"{pw}.bias"] = g.normal((cin,), 0.05)


def roma_weights(seed=0):
    """(main, dino, v2) state_dicts of RoMa outdoor, DINOv2 ViT-L/14 and
    RoMa v2's refiners, seeded random init (BatchNorm statistics
    randomized)."""
    g = Gen(seed)
    main, dino, v2 = {}, {}, {}
    _vgg(g, main, "encoder.cnn.layers", 4)
    dino["patch_embed.proj.weight"] = g.normal((VIT_DIM, 3, 14, 14), 0.02)
    dino["patch_embed.proj.bias"] = g.normal((VIT_DIM,), 0.02)
    dino["cls_token"] = g.normal((1, 1, VIT_DIM), 0.02)
    dino["pos_embed"] = g.normal((1, 37 * 37 + 1, VIT_DIM), 0.02)
    for i in range(VIT_DEPTH):
        _block(g, dino, f"blocks.{i}", VIT_DIM, True, g.uniform((VIT_DIM,), 0.05, 0.15))
    dino["norm.weight"] = 1.0 + g.normal((VIT_DIM,), 0.02)
    dino["norm.bias"] = g.normal((VIT_DIM,), 0.02)
    for s in range(5):
        f, pin = REF_FEAT[s], PROJ_IN[s]
        pre = f"decoder.proj.{REF_SCALE[s]}"
        main[f"{pre}.0.weight"] = g.normal((f, pin, 1, 1), math.sqrt(1.0 / pin))
        main[f"{pre}.0.bias"] = g.normal((f,), 0.05)
        _bn(g, main, f"{pre}.1", f)
    main["decoder.gps.16.pos_conv.weight"] = g.uniform((512, 2, 1, 1), -0.7071, 0.7071)
    main["decoder.gps.16.pos_conv.bias"] = g.uniform((512,), -0.7071, 0.7071)
    for i in range(DEC_DEPTH):
        _block(g, main, f"decoder.embedding_decoder.blocks.{i}", VIT_DIM, False, None)
    main["decoder.embedding_decoder.to_out.weight"] = g.normal((64 * 64 + 1, VIT_DIM), 0.02)
    main["decoder.embedding_decoder.to_out.bias"] = g.normal((64 * 64 + 1,), 0.02)
    for s in range(5):
        f, e, r = REF_FEAT[s], REF_EMB[s], REF_RADIUS[s]
        cin = 2 * f + e + ((2 * r + 1) ** 2 if r else 0)
        pre = f"decoder.conv_refiner.{REF_SCALE[s]}"
        _ref_blocks(g, main, pre, cin, False)
        main[f"{pre}.out_conv.weight"] = g.normal((3, cin, 1, 1), math.sqrt(1.0 / cin))
        main[f"{pre}.out_conv.bias"] = g.normal((3,), 0.05)
        main[f"{pre}.disp_emb.weight"] = g.normal((e, 2, 1, 1), 0.7)
        main[f"{pre}.disp_emb.bias"] = g.normal((e,), 0.05)
    _roma_v2(g, v2)
    return main, dino, v2


def roma_v2_weights(seed=0):
    """RoMa v2's refiners alone (their own seeded stream, not the one
    roma_weights draws them from)."""
    v2 = {}
    _roma_v2(Gen(seed), v2)
    return v2


def _roma_v2(g, v2):
    """RoMa v2's refiner features and refiners (roma.c:460-545)."""
    _vgg(g, v2, "refiner_features.layers", 3)
    for j in range(3):
        f, e, r, fin = REF2_FEAT[j], REF2_EMB[j], REF2_RADIUS[j], REF2_IN[j]
        cin = 2 * f + e + ((2 * r + 1) ** 2 if r else 0)
        pre = f"refiners.{REF2_SCALE[j]}"
        v2[f"{pre}.proj.weight"] = g.normal((f, fin), math.sqrt(1.0 / fin))
        v2[f"{pre}.proj.bias"] = g.normal((f,), 0.05)
        _ref_blocks(g, v2, pre, cin, True)
        v2[f"{pre}.disp_emb.weight"] = g.normal((e, 2, 1, 1), 0.7)
        v2[f"{pre}.disp_emb.bias"] = g.normal((e,), 0.05)
        v2[f"{pre}.warp_head.weight"] = g.normal((2, cin, 1, 1), math.sqrt(1.0 / cin))
        v2[f"{pre}.warp_head.bias"] = g.normal((2,), 0.05)
        v2[f"{pre}.confidence_head.weight"] = g.normal((4, cin, 1, 1), math.sqrt(1.0 / cin))
        v2[f"{pre}.confidence_head.bias"] = g.normal((4,), 0.05)


def write_roma_weights(folder, seed=0):
    """Write roma_main / dino / v2 safetensors into folder; returns the
    three paths."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    paths = []
    for name, sd in zip(("roma_main", "dinov2", "romav2_refiners"), roma_weights(seed)):
        p = folder / f"{name}_seed{seed}.safetensors"
        if not p.exists():
            tmp = p.with_suffix(".tmp")
            write_safetensors(tmp, sd)
            tmp.rename(p)
        paths.append(p)
    return paths


# DISK's U-Net (disk.c:23-31): input and output channels per layer.
DISK_CIN = (3, 16, 32, 64, 64, 128, 128, 96, 80)
DISK_COUT = (16, 32, 64, 64, 64, 64, 64, 64, 129)


def disk_weights(seed=0):
    """Seeded random-init DISK U-Net in the extractor state_dict names the
    loader requires ("unet.path_down.{0..4}.1.{1,3}",
    "unet.path_up.{0..3}.conv.{1,3}"): convolutions He-normal, biases
    N(0, 0.01), PReLU slopes 0.25 + N(0, 0.02)."""
    g = np.random.default_rng(seed)
    d = {}
    for l, (ci, co) in enumerate(zip(DISK_CIN, DISK_COUT)):
        pre = f"unet.path_down.{l}.1" if l < 5 else f"unet.path_up.{l - 5}.conv"
        d[f"{pre}.3.weight"] = (g.standard_normal((co, ci, 5, 5)) *
                                math.sqrt(2.0 / (ci * 25))).astype(np.float32)
        d[f"{pre}.3.bias"] = (0.01 * g.standard_normal(co)).astype(np.float32)
        if l > 0:
            d[f"{pre}.1.weight"] = (0.25 + 0.02 * g.standard_normal(ci)).astype(np.float32)
    return d


def write_disk_weights(folder, seed=0):
    """Write the DISK weights as safetensors into folder; returns the path."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    p = folder / f"disk_seed{seed}.safetensors"
    if not p.exists():
        tmp = p.with_suffix(".tmp")
        write_safetensors(tmp, disk_weights(seed))
        tmp.rename(p)
    return p


def eloftr_weights(seed=0):
    """Seeded random-init Efficient LoFTR in the names of
    EfficientLoFTRForKeypointMatching (what the loader requires): RepVGG
    backbone (3 x 3, 1 x 1 and identity branches with BatchNorms), the
    aggregated-attention transformer, the fine fusion. Scales keep the
    activations bounded through the 21 blocks."""
    g = np.random.default_rng(seed)
    d = {}
    n = lambda *s_, std=1.0: (std * g.standard_normal(s_)).astype(np.float32)

    def bn(pre, c, gain=1.0):
        d[f"{pre}.weight"] = (gain * (1.0 + 0.1 * g.standard_normal(c))).astype(np.float32)
        d[f"{pre}.bias"] = n(c, std=0.1)
        d[f"{pre}.running_mean"] = n(c, std=0.1)
        d[f"{pre}.running_var"] = g.uniform(0.5, 1.5, c).astype(np.float32)

    cin = 1
    for s_, (nb, co, st) in enumerate(zip((1, 2, 4, 14), (64, 64, 128, 256), (2, 1, 2, 2))):
        for b in range(nb):
            stride = st if b == 0 else 1
            pre = f"efficientloftr.backbone.stages.{s_}.blocks.{b}"
            gain = 1.0
            d[f"{pre}.conv1.conv.weight"] = n(co, cin, 3, 3, std=0.5 * math.sqrt(2.0 / (9 * cin)))
            bn(f"{pre}.conv1.norm", co, gain)
            d[f"{pre}.conv2.conv.weight"] = n(co, cin, 1, 1, std=0.5 * math.sqrt(2.0 / cin))
            bn(f"{pre}.conv2.norm", co, gain)
            if cin == co and stride == 1:
                bn(f"{pre}.identity", co, gain)
            cin = co
    D, M = 256, 512
    for l in range(4):
        for kind in ("self_attention", "cross_attention"):
            pre = f"efficientloftr.local_feature_transformer.layers.{l}.{kind}."
            d[pre + "aggregation.q_aggregation.weight"] = n(D, 1, 4, 4, std=0.25)
            d[pre + "aggregation.norm.weight"] = (1.0 + 0.1 * g.standard_normal(D)).astype(np.float32)
            d[pre + "aggregation.norm.bias"] = n(D, std=0.1)
            for p in ("q", "k", "v", "o"):
                d[pre + f"attention.{p}_proj.weight"] = n(D, D, std=1.0 / math.sqrt(D))
            d[pre + "mlp.fc1.weight"] = n(M, 2 * D, std=math.sqrt(2.0 / (2 * D)))
            d[pre + "mlp.fc2.weight"] = n(D, M, std=1.0 / math.sqrt(M))
            d[pre + "mlp.layer_norm.weight"] = (1.0 + 0.1 * g.standard_normal(D)).astype(np.float32)
            d[pre + "mlp.layer_norm.bias"] = n(D, std=0.1)
    d["refinement_layer.out_conv.weight"] = n(256, 256, 1, 1, std=1.0 / 16)
    for i, (hid, inter) in enumerate(((128, 256), (64, 128))):
        pre = f"refinement_layer.out_conv_layers.{i}."
        d[pre + "out_conv1.weight"] = n(inter, hid, 1, 1, std=1.0 / math.sqrt(hid))
        d[pre + "out_conv2.weight"] = n(inter, inter, 3, 3, std=math.sqrt(2.0 / (9 * inter)))
        bn(pre + "batch_norm", inter)
        d[pre + "out_conv3.weight"] = n(hid, inter, 3, 3, std=1.0 / math.sqrt(9 * inter))
    return d


def write_eloftr_weights(folder, seed=0):
    """Write the Efficient LoFTR weights as safetensors; returns the path."""
    folder = Path(folder)
    folder.mkdir(parents=True, exist_ok=True)
    p = folder / f"eloftr_seed{seed}.safetensors"
    if not p.exists():
        tmp = p.with_suffix(".tmp")
        write_safetensors(tmp, eloftr_weights(seed))
        tmp.rename(p)
    return p


# ----------------------------------------------------------------- images

def band_limited(rng, h, w, sigma, mean=128.0, std=40.0):
    """Gaussian-filtered N(mean, std) noise, clipped to 0..255 (the
    benchmark configurations' 'band-limited noise'), float64."""
    from scipy.ndimage import gaussian_filter

    x = rng.normal(mean, std, (h, w))
    x = gaussian_filter(x, sigma, mode="wrap")
    # Restore the contrast the filter removed.
    x = (x - x.mean()) / max(x.std(), 1e-9) * std + mean
    return np.clip(x, 0, 255)


def warp_bilinear(img, mapx, mapy):
    """Sample img (C, H, W) at float pixel coordinates (bilinear, edge
    clamp)."""
    from scipy.ndimage import map_coordinates

    return np.stack([map_coordinates(c, [mapy, mapx], order=1, mode="nearest") for c in img])


def scene_pair(seed, H, W, bands=3, sigma=3.0, drift=12.0, patches=64):
    """Config-4-style pair: reference = band-limited noise with seeded
    piecewise-constant rectangles; target = reference under an affine plus
    smooth sinusoidal drift (<= drift px), per-band gain 0.8..1.2, N(0, 4)
    noise. uint8 (bands, H, W) each, and the true map (x, y) of target
    pixels into the reference."""
    rng = np.random.default_rng(seed)
    ref = np.stack([band_limited(rng, H, W, sigma) for _ in range(bands)])
    for _ in range(patches):
        h, w = rng.integers(32, max(33, min(512, H // 2)), 2)
        y, x = rng.integers(0, max(1, H - h)), rng.integers(0, max(1, W - w))
        ref[:, y:y + h, x:x + w] = rng.uniform(20, 235, (bands, 1, 1))
    yy, xx = np.mgrid[0:H, 0:W].astype(np.float64)
    ang = np.deg2rad(rng.uniform(-2, 2))
    sc = rng.uniform(0.98, 1.02)
    cx, cy = W / 2, H / 2
    mx = cx + sc * (np.cos(ang) * (xx - cx) - np.sin(ang) * (yy - cy)) + rng.uniform(-10, 10)
    my = cy + sc * (np.sin(ang) * (xx - cx) + np.cos(ang) * (yy - cy)) + rng.uniform(-10, 10)
    for _ in range(2):
        kx, ky = rng.uniform(0.5, 2.0, 2) * 2 * np.pi / max(H, W)
        ph = rng.uniform(0, 2 * np.pi, 2)
        mx += drift / 2 * np.sin(kx * xx + ky * yy + ph[0])
        my += drift / 2 * np.cos(ky * xx - kx * yy + ph[1])
    tgt = warp_bilinear(ref, mx, my)
    tgt *= rng.uniform(0.8, 1.2, (bands, 1, 1))
    tgt += rng.normal(0, 4, tgt.shape)
    return (np.clip(ref, 0, 255).astype(np.uint8), np.clip(tgt, 0, 255).astype(np.uint8),
            np.stack([mx, my]))


def grey_affine_pair(seed, H, W):
    """Config-2 pair (Efficient LoFTR): A = band-limited noise (N(128, 40),
    Gaussian sigma 3 px, clipped) from seed; B = A under a seeded affine
    (rotation within 5 degrees, scale 0.95..1.05, shift within 20 px, from
    seed + 1) plus N(0, 3) noise. uint8 (H, W) each."""
    rng = np.random.default_rng(seed)
    a = band_limited(rng, H, W, 3.0)
    r = np.random.default_rng(seed + 1)
    ang = np.deg2rad(r.uniform(-5, 5))
    sc = r.uniform(0.95, 1.05)
    tx, ty = r.uniform(-20, 20, 2)
    yy, xx = np.mgrid[0:H, 0:W].astype(np.float64)
    cx, cy = W / 2, H / 2
    mx = cx + sc * (np.cos(ang) * (xx - cx) - np.sin(ang) * (yy - cy)) + tx
    my = cy + sc * (np.sin(ang) * (xx - cx) + np.cos(ang) * (yy - cy)) + ty
    b = warp_bilinear(a[None], mx, my)[0] + r.normal(0, 3, (H, W))
    return np.clip(a, 0, 255).astype(np.uint8), np.clip(b, 0, 255).astype(np.uint8)


def tile_input(img_u8, H, W):
    """uint8 (3, h, w) tile to the matcher input: (3, H, W) float32 in
    0..1, zero padded (the reference's tile_input, main.c)."""
    c, h, w = img_u8.shape
    out = np.zeros((3, H, W), np.float32)
    out[:c, :h, :w] = img_u8.astype(np.float32) / 255.0
    return out
