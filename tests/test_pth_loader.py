# SPDX-License-Identifier: Unlicense
"""The weight-file reader of the C-ABI library (include/pth_loader.h, the
reference's pth_loader.c) against torch.load: every float tensor that
torch.load returns for a checkpoint comes back from pth_read_f32
bit-exact, with its name, shape and order, for the formats the reference
reads (torch.save zip archives in pickle protocols 2 and 4 and in zip64
form, the legacy torch.save stream, safetensors), for views (transposed,
sliced, sharing a storage), parameters and tensors with Python
attributes, and for the wrappers around a state_dict the reference
accepts ("model", "state_dict", a single dict of tensors). Integer
tensors are left out. Malformed files give the reference's errors.

The well-formed files are also read by the reference's own pth_loader.c,
compiled into oracle/_ref/libpth_ref.so by oracle/Makefile (that test
skips when it has not been built): the same index (names, shapes, strides,
storage offsets, dtypes, file offsets, storage sizes), the same pth_bytes
and bit-identical pth_read_f32 arrays. CPU only: no device call."""

import ctypes as C
import io
import json
import struct
import zipfile
from collections import OrderedDict
from pathlib import Path

import numpy as np
import pytest
import torch

import coreg
from coreg import roma as R
from coreg import synth

LIBC = C.CDLL(None)
LIBC.free.argtypes = [C.c_void_p]


@pytest.fixture()
def lib():
    lib = coreg.load()
    lib.coreg_set_error_mode(coreg.ERRORS_RECORD)
    lib.coreg_clear_error()
    yield lib
    lib.coreg_clear_error()
    lib.coreg_set_error_mode(coreg.ERRORS_FATAL)


def open_pth(lib, path):
    pf = R.PthFile()
    lib.pth_open(C.byref(pf), str(path).encode())
    err = lib.coreg_last_error()
    if err:
        lib.coreg_clear_error()
        return None, err.decode()
    return pf, None


def read_all(lib, path):
    """OrderedDict name -> float32 array of everything pth_open indexed."""
    pf, err = open_pth(lib, path)
    assert err is None, err
    out = OrderedDict()
    try:
        for i in range(pf.ntensors):
            t = pf.tensors[i]
            shape = tuple(t.shape[:t.ndim])
            p = lib.pth_read_f32(C.byref(pf), C.byref(t))
            assert p and not lib.coreg_last_error()
            n = int(np.prod(shape))
            a = np.ctypeslib.as_array(p, (max(n, 1),))[:n].copy().reshape(shape)
            LIBC.free(C.cast(p, C.c_void_p))
            out[t.name.decode()] = a
    finally:
        lib.pth_close(C.byref(pf))
    return out


def expected(sd):
    """The float tensors of a state_dict, as torch.load gives them."""
    return OrderedDict((k, v.detach().float().numpy()) for k, v in sd.items()
                       if torch.is_tensor(v) and v.dtype in (torch.float32, torch.float16,
                                                             torch.bfloat16))


def assert_same(got, want):
    assert list(got) == list(want)
    for k in want:
        assert got[k].shape == want[k].shape, k
        assert np.array_equal(got[k].view(np.uint32), want[k].view(np.uint32)), k


def state_dict():
    g = torch.Generator().manual_seed(3)
    base = torch.randn(6, 5, generator=g)
    shared = torch.randn(40, generator=g)
    tagged = torch.randn(7, generator=g)
    tagged.note = "attr"  # pickled through torch._tensor._rebuild_from_type_v2
    half = torch.randn(3, 2, generator=g).half()
    half[0, 0] = 6.0e-8  # a float16 subnormal
    half[0, 1] = -65504.0
    return OrderedDict([
        ("enc.conv.weight", torch.randn(8, 3, 3, 3, generator=g)),
        ("enc.conv.bias", torch.randn(8, generator=g)),
        ("enc.bn.num_batches_tracked", torch.tensor(17)),
        ("enc.half", half),
        ("enc.bf16", torch.randn(4, 3, generator=g).bfloat16()),
        ("view.t", base.t()),
        ("view.rows", base[2:5]),
        ("view.cols", base[:, 1:4]),
        ("view.shared_a", shared[:12].view(3, 4)),
        ("view.shared_b", shared[20:40:2]),
        ("scalar", torch.tensor(2.5)),
        ("param", torch.nn.Parameter(torch.randn(2, 2, generator=g))),
        ("tagged", tagged),
        ("mask", torch.ones(3, dtype=torch.bool)),
        ("ids", torch.arange(5, dtype=torch.int32)),
    ])


@pytest.mark.parametrize("how", ["zip", "zip_protocol4", "legacy"])
def test_torch_save_formats_match_torch_load(lib, tmp_path, how):
    sd = state_dict()
    p = tmp_path / "w.pth"
    if how == "zip":
        torch.save(sd, p)
    elif how == "zip_protocol4":
        torch.save(sd, p, pickle_protocol=4)
    else:
        torch.save(sd, p, _use_new_zipfile_serialization=False)
    want = expected(torch.load(p, weights_only=False))
    assert "enc.bn.num_batches_tracked" not in want and "ids" not in want
    got = read_all(lib, p)
    assert_same(got, want)


def test_archive_folder_name_from_a_stream(lib, tmp_path):
    """torch.save to a stream names the archive's folder "archive/"; the
    reader finds data.pkl and the storages under any folder name."""
    buf = io.BytesIO()
    sd = state_dict()
    torch.save(sd, buf)
    p = tmp_path / "stream.pth"
    p.write_bytes(buf.getvalue())
    with zipfile.ZipFile(p) as z:
        assert any(n.startswith("archive/") for n in z.namelist())
    assert_same(read_all(lib, p), expected(torch.load(p, weights_only=False)))


def test_views_keep_their_strides(lib, tmp_path):
    sd = state_dict()
    p = tmp_path / "w.pth"
    torch.save(sd, p)
    pf, err = open_pth(lib, p)
    assert err is None
    try:
        by = {pf.tensors[i].name.decode(): pf.tensors[i] for i in range(pf.ntensors)}
        t = by["view.t"]
        assert list(t.shape[:2]) == [5, 6] and list(t.stride[:2]) == [1, 5]
        assert by["view.rows"].storage_offset == 10
        assert by["view.shared_b"].storage_offset == 20 and by["view.shared_b"].stride[0] == 2
        assert by["scalar"].ndim == 0
        assert by["enc.half"].dtype == R.PTH_F16 and by["enc.bf16"].dtype == R.PTH_BF16
        # pth_bytes counts the tensors' own elements, not their storages.
        want = sum(v.numel() * v.element_size() for k, v in sd.items()
                   if k.startswith("view.") and v.dtype == torch.float32)
        assert lib.pth_bytes(C.byref(pf), b"view.") == want
    finally:
        lib.pth_close(C.byref(pf))


def zip64_copy(src, dst):
    """The same archive rewritten with zip64 records everywhere (sizes,
    offsets and the end-of-directory record past their 32-bit fields)."""
    old = zipfile.ZIP64_LIMIT, zipfile.ZIP_FILECOUNT_LIMIT
    zipfile.ZIP64_LIMIT, zipfile.ZIP_FILECOUNT_LIMIT = 0, 0
    try:
        with zipfile.ZipFile(src) as zi, zipfile.ZipFile(dst, "w", zipfile.ZIP_STORED) as zo:
            for info in zi.infolist():
                zo.writestr(info.filename, zi.read(info.filename))
    finally:
        zipfile.ZIP64_LIMIT, zipfile.ZIP_FILECOUNT_LIMIT = old
    raw = open(dst, "rb").read()
    assert b"PK\x06\x06" in raw and b"PK\x06\x07" in raw


def test_zip64_archive(lib, tmp_path):
    sd = state_dict()
    src, dst = tmp_path / "w.pth", tmp_path / "w64.pth"
    torch.save(sd, src)
    zip64_copy(src, dst)
    assert_same(read_all(lib, dst), expected(torch.load(dst, weights_only=False)))


@pytest.mark.parametrize("wrap", ["model", "state_dict", "extractor"])
def test_state_dict_wrappers(lib, tmp_path, wrap):
    sd = state_dict()
    obj = {"epoch": 3, "meta": {"lr": 0.1}, wrap: sd}
    if wrap == "model":
        obj["optimizer"] = {"state": {}, "lr": 1e-3}
    p = tmp_path / "w.pth"
    torch.save(obj, p)
    assert_same(read_all(lib, p), expected(sd))


def test_ambiguous_wrapper_is_refused(lib, tmp_path):
    p = tmp_path / "w.pth"
    torch.save({"a": {"x": torch.zeros(2)}, "b": {"y": torch.zeros(2)}}, p)
    pf, err = open_pth(lib, p)
    assert pf is None and "No state_dict" in err


def test_prefix_strip_of_wrapped_names(lib, tmp_path):
    p = tmp_path / "w.pth"
    torch.save({"matcher.model.a": torch.ones(2), "matcher.model.b": torch.ones(3),
                "other": torch.ones(1)}, p)
    pf, err = open_pth(lib, p)
    assert err is None
    try:
        assert lib.pth_strip_prefix(C.byref(pf), b"matcher.model.") == 2
        names = [pf.tensors[i].name.decode() for i in range(pf.ntensors)]
        assert names == ["a", "b", "other"]
        assert lib.pth_find(C.byref(pf), b"a")
    finally:
        lib.pth_close(C.byref(pf))


def write_safetensors_mixed(path):
    g = np.random.default_rng(4)
    f32 = g.standard_normal((3, 4)).astype(np.float32)
    f16 = g.standard_normal(5).astype(np.float16)
    bf16 = (g.standard_normal(6).astype(np.float32).view(np.uint32) >> 16).astype(np.uint16)
    i64 = np.arange(3, dtype=np.int64)
    parts = [("w", "F32", f32), ("h", "F16", f16), ("b", "BF16", bf16), ("n", "I64", i64)]
    header, off, blobs = {"__metadata__": {"format": "pt"}}, 0, []
    for name, dt, a in parts:
        header[name] = {"dtype": dt, "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
        blobs.append(a.tobytes())
    h = json.dumps(header).encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(h)) + h + b"".join(blobs))
    return OrderedDict([("w", f32), ("h", f16.astype(np.float32)),
                        ("b", (bf16.astype(np.uint32) << 16).view(np.float32))])


def test_safetensors(lib, tmp_path):
    p = tmp_path / "w.safetensors"
    want = write_safetensors_mixed(p)
    assert_same(read_all(lib, p), want)


def test_disk_weights_read_the_same_from_pth_and_safetensors(lib, tmp_path):
    """DISK's checkpoint holds its weights under "extractor"; the loader
    gives disk_load the same arrays from either format."""
    w = synth.disk_weights(0)
    st = tmp_path / "disk.safetensors"
    synth.write_safetensors(st, dict(w))
    pth = tmp_path / "disk.pth"
    torch.save({"extractor": OrderedDict((k, torch.from_numpy(np.asarray(v, np.float32)))
                                         for k, v in w.items())}, pth)
    a, b = read_all(lib, st), read_all(lib, pth)
    assert sorted(a) == sorted(b) and len(a) == len(w)
    for k in a:
        assert np.array_equal(a[k], b[k]), k


def test_malformed_files(lib, tmp_path):
    cases = {}
    # A deflated data.pkl: torch.save writes stored entries only.
    good = tmp_path / "good.pth"
    torch.save({"x": torch.ones(3)}, good)
    deflated = tmp_path / "deflated.pth"
    with zipfile.ZipFile(good) as zi, zipfile.ZipFile(deflated, "w", zipfile.ZIP_DEFLATED) as zo:
        for info in zi.infolist():
            zo.writestr(info.filename, zi.read(info.filename))
    cases[deflated] = "compressed"
    nopkl = tmp_path / "nopkl.pth"
    with zipfile.ZipFile(nopkl, "w") as zo:
        zo.writestr("w/data/0", b"\0" * 12)
    cases[nopkl] = "No data.pkl"
    raw = good.read_bytes()
    truncated = tmp_path / "truncated.pth"
    truncated.write_bytes(raw[: len(raw) // 2])
    cases[truncated] = "zip"
    junk = tmp_path / "junk.bin"
    junk.write_bytes(bytes(range(7, 207)))
    cases[junk] = "not a PyTorch checkpoint"
    short = tmp_path / "short.pth"
    short.write_bytes(b"PK")
    cases[short] = "too short"
    # A storage entry shorter than its tensor.
    small = tmp_path / "small.pth"
    with zipfile.ZipFile(good) as zi, zipfile.ZipFile(small, "w") as zo:
        for info in zi.infolist():
            data = zi.read(info.filename)
            zo.writestr(info.filename, data[:4] if info.filename.endswith("data/0") else data)
    cases[small] = "exceeds its storage"
    # An opcode outside what a state_dict pickles to (a pickled set of
    # ints is fine; PERSID in text form is not).
    odd = tmp_path / "odd.pth"
    with zipfile.ZipFile(odd, "w") as zo:
        zo.writestr("w/data.pkl", b"\x80\x02Pabc\n.")
    cases[odd] = "opcode"
    missing = tmp_path / "absent.pth"
    cases[missing] = "Unable to open"
    for path, msg in cases.items():
        pf, err = open_pth(lib, path)
        assert pf is None and err is not None and msg in err, (path.name, err)
    # The recorded error leaves the next open unaffected.
    assert read_all(lib, good)["x"].tolist() == [1.0, 1.0, 1.0]


def test_missing_tensor_and_wrong_shape(lib, tmp_path):
    p = tmp_path / "w.pth"
    torch.save({"x": torch.ones(2, 3)}, p)
    pf, err = open_pth(lib, p)
    assert err is None
    try:
        shape = (C.c_long * 2)(2, 4)
        assert not lib.pth_require(C.byref(pf), b"x", 2, shape)
        assert "along axis 1" in lib.coreg_last_error().decode()
        lib.coreg_clear_error()
        assert not lib.pth_require(C.byref(pf), b"y", 2, None)
        assert "not found" in lib.coreg_last_error().decode()
        lib.coreg_clear_error()
        shape = (C.c_long * 2)(2, -1)
        t = lib.pth_require(C.byref(pf), b"x", 2, shape)
        assert t and lib.pth_numel(t) == 6
    finally:
        lib.pth_close(C.byref(pf))


PTH_REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libpth_ref.so"


@pytest.fixture(scope="module")
def ref_reader():
    if not PTH_REF.exists():
        pytest.skip("oracle/_ref/libpth_ref.so not built (make -C oracle)")
    r = C.CDLL(str(PTH_REF))
    r.pth_open.restype = None
    r.pth_open.argtypes = [C.POINTER(R.PthFile), C.c_char_p]
    r.pth_read_f32.restype = C.POINTER(C.c_float)
    r.pth_read_f32.argtypes = [C.POINTER(R.PthFile), C.POINTER(R.PthTensor)]
    r.pth_bytes.restype = C.c_double
    r.pth_bytes.argtypes = [C.POINTER(R.PthFile), C.c_char_p]
    r.pth_close.restype = None
    r.pth_close.argtypes = [C.POINTER(R.PthFile)]
    return r


def index_and_data(lib, path, prefix=b""):
    """(index rows, arrays, pth_bytes(prefix)) of a reader: this build's
    library or the reference's."""
    pf = R.PthFile()
    lib.pth_open(C.byref(pf), str(path).encode())
    rows, arrays = [], []
    for i in range(pf.ntensors):
        t = pf.tensors[i]
        rows.append((t.name.decode(), t.ndim, tuple(t.shape[:t.ndim]), tuple(t.stride[:t.ndim]),
                     t.storage_offset, t.dtype, t.data_offset, t.storage_bytes))
        p = lib.pth_read_f32(C.byref(pf), C.byref(t))
        n = int(np.prod(t.shape[:t.ndim]))
        arrays.append(np.ctypeslib.as_array(p, (max(n, 1),))[:n].copy())
        LIBC.free(C.cast(p, C.c_void_p))
    nbytes = lib.pth_bytes(C.byref(pf), prefix)
    lib.pth_close(C.byref(pf))
    return rows, arrays, nbytes


def well_formed_files(tmp_path):
    sd = state_dict()
    files = {}
    for name, kw in (("zip", {}), ("p4", {"pickle_protocol": 4}),
                     ("legacy", {"_use_new_zipfile_serialization": False})):
        files[name] = tmp_path / f"{name}.pth"
        torch.save(sd, files[name], **kw)
    files["zip64"] = tmp_path / "z64.pth"
    zip64_copy(files["zip"], files["zip64"])
    files["wrapped"] = tmp_path / "wrapped.pth"
    torch.save({"epoch": 1, "model": sd}, files["wrapped"])
    buf = io.BytesIO()
    torch.save(sd, buf)
    files["stream"] = tmp_path / "stream.pth"
    files["stream"].write_bytes(buf.getvalue())
    files["safetensors"] = tmp_path / "w.safetensors"
    write_safetensors_mixed(files["safetensors"])
    return files


def test_index_and_values_match_reference_reader(lib, ref_reader, tmp_path):
    for name, path in well_formed_files(tmp_path).items():
        mine = index_and_data(lib, path, b"view.")
        ref = index_and_data(ref_reader, path, b"view.")
        assert mine[0] == ref[0], name
        assert mine[2] == ref[2], name
        for a, b in zip(mine[1], ref[1]):
            assert np.array_equal(a.view(np.uint32), b.view(np.uint32)), name
