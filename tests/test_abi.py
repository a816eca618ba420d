"""C ABI: the library loads, exports every declared symbol, and its host-only
SafeTensors check mirrors the reference loader's tests
(crates/weight_loader/src/safe_tensors.rs:140-236, mmap.rs:168-242).
No GPU compute is called here."""
import json
import os
import re
import struct

import numpy as np
import pytest

import myos
from myos import _lib

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.fixture(scope="module", autouse=True)
def built():
    import build as pkg_build

    pkg_build.build()


def declared_symbols():
    text = open(os.path.join(REPO, "include", "myos_cuda.h")).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(myos_[a-z0-9_]+)\s*\(", text)))


def test_every_declared_symbol_is_exported():
    L = _lib.load()
    names = declared_symbols()
    assert len(names) >= 20
    for n in names:
        assert hasattr(L, n), n
    assert set(names) == set(_lib.SIGNATURES), "binding table and header disagree"


def test_version_and_shapes_need_no_gpu():
    L = _lib.load()
    assert b"sm_100a" in L.myos_version()
    s = L.myos_shape_qwen25_1_5b().as_dict()
    assert s["hidden"] == 1536 and s["num_layers"] == 28 and s["vocab"] == 151936
    assert s["num_q_heads"] == 12 and s["num_kv_heads"] == 2 and s["head_dim"] == 128
    assert s["intermediate"] == 8960 and s["tied_head"] == 1
    assert np.float32(s["rms_eps"]) == np.float32(1e-6) and s["rope_theta"] == 1e6
    b = L.myos_shape_qwen25_14b().as_dict()
    assert b["hidden"] == 5120 and b["num_layers"] == 48 and b["tied_head"] == 0


def test_tensor_parallel_split_is_checked_before_any_device_work():
    """myos_ctx_create_tp refuses splits that do not divide the model (and
    bad ranks) from the shape alone: no GPU, no NCCL."""
    import ctypes as C
    L = _lib.load()
    opts = _lib.Opts(0, 64, _lib.KV_F32, 1)

    def create(shape, size, rank):
        t = _lib.TP(size, rank)
        h = C.c_void_p()
        return L.myos_ctx_create_tp(C.byref(shape), C.byref(opts), C.byref(t), C.byref(h))

    small = L.myos_shape_qwen25_1_5b()  # 12 q heads, 2 kv heads
    big = L.myos_shape_qwen25_14b()     # 40 q heads, 8 kv heads, head_dim 128
    assert create(small, 4, 0) == _lib.ERR_SHAPE   # 2 kv heads over 4 ranks
    assert create(small, 3, 0) == _lib.ERR_SHAPE   # 2 kv heads over 3 ranks
    assert create(big, 3, 0) == _lib.ERR_SHAPE     # 40 q heads over 3 ranks
    assert create(big, 16, 0) == _lib.ERR_ARG      # more than 8 ranks
    assert create(small, 2, 2) == _lib.ERR_ARG     # rank out of range
    assert create(small, 0, 0) == _lib.ERR_ARG
    assert C.sizeof(_lib.TP) == 136


def _write(path, entries, pad=True, metadata=None):
    header = {}
    off = 0
    blobs = []
    for name, dtype, shape, data in entries:
        header[name] = {"dtype": dtype, "shape": shape, "data_offsets": [off, off + len(data)]}
        off += len(data)
        blobs.append(data)
    if metadata is not None:
        header["__metadata__"] = metadata
    hb = json.dumps(header).encode()
    if pad:
        hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)) + hb + b"".join(blobs))


def test_parses_f32_f16_bf16(tmp_path):
    p = str(tmp_path / "ok.safetensors")
    _write(p, [("w_f32", "F32", [2], np.array([1.0, -2.5], "<f4").tobytes()),
               ("w_f16", "F16", [2], bytes([0x00, 0x3C, 0x00, 0xC0])),
               ("w_bf16", "BF16", [1, 2], bytes([0x80, 0x3F, 0x00, 0xC0])),
               ("bias", "F32", [], np.array([0.5], "<f4").tobytes())], metadata={"k": "v"})
    assert myos.check_safetensors(p) == 4


def test_rejects_unmapped_dtype_for_the_whole_file(tmp_path):
    p = str(tmp_path / "i64.safetensors")
    _write(p, [("keep", "F32", [1], np.array([1.0], "<f4").tobytes()),
               ("drop", "I64", [1], np.array([7], "<i8").tobytes())])
    with pytest.raises(myos.MyosError) as e:
        myos.check_safetensors(p)
    assert e.value.code == _lib.ERR_UNSUPPORTED


@pytest.mark.parametrize("blob", [b"", b"short", bytes([0xFF, 0, 0, 0, 0, 0, 0, 0]),
                                  bytes([0xFF] * 8)])
def test_rejects_truncated_buffers(tmp_path, blob):
    p = str(tmp_path / "bad.safetensors")
    open(p, "wb").write(blob)
    with pytest.raises(myos.MyosError) as e:
        myos.check_safetensors(p)
    assert e.value.code == _lib.ERR_PARSE


def test_rejects_gaps_overlaps_and_bad_lengths(tmp_path):
    data = np.arange(4, dtype="<f4").tobytes()
    good = {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
            "b": {"dtype": "F32", "shape": [2], "data_offsets": [8, 16]}}
    cases = [
        {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]},
         "b": {"dtype": "F32", "shape": [2], "data_offsets": [12, 20]}},  # gap
        {"a": {"dtype": "F32", "shape": [3], "data_offsets": [0, 8]},
         "b": {"dtype": "F32", "shape": [2], "data_offsets": [8, 16]}},  # length
        {"a": {"dtype": "F32", "shape": [2], "data_offsets": [0, 8]}},    # trailing bytes
        {"a": {"dtype": "Q7", "shape": [2], "data_offsets": [0, 8]},
         "b": {"dtype": "F32", "shape": [2], "data_offsets": [8, 16]}},  # unknown tag
    ]
    p = str(tmp_path / "g.safetensors")
    hb = json.dumps(good).encode()
    open(p, "wb").write(struct.pack("<Q", len(hb)) + hb + data)
    assert myos.check_safetensors(p) == 2
    for i, hdr in enumerate(cases):
        p = str(tmp_path / f"c{i}.safetensors")
        hb = json.dumps(hdr).encode()
        open(p, "wb").write(struct.pack("<Q", len(hb)) + hb + data)
        with pytest.raises(myos.MyosError) as e:
            myos.check_safetensors(p)
        assert e.value.code == _lib.ERR_PARSE, i


def test_missing_file_is_io(tmp_path):
    with pytest.raises(myos.MyosError) as e:
        myos.check_safetensors(str(tmp_path / "nope.safetensors"))
    assert e.value.code == _lib.ERR_IO


def test_writer_roundtrip_matches_python_safetensors(tmp_path):
    from myos import synth
    st = pytest.importorskip("safetensors.numpy")
    table = {"x": ((2, 3), np.arange(6, dtype=np.uint16).view(np.uint8)),
             "y": ((4,), np.arange(4, dtype=np.uint16).view(np.uint8))}
    p = str(tmp_path / "w.safetensors")
    synth.write_safetensors(p, table, {"seed": 7})
    assert myos.check_safetensors(p) == 2
    # the reference fixtures are written by the safetensors crate; its Python
    # twin must read ours and ours must read its output
    from safetensors import safe_open
    with safe_open(p, "np") as f:
        assert sorted(f.keys()) == ["x", "y"]
    q = str(tmp_path / "theirs.safetensors")
    st.save_file({"a": np.ones((3, 2), np.float32)}, q)
    assert myos.check_safetensors(q) == 1


def test_struct_layouts_match_the_header(tmp_path):
    """myos_shape / myos_opts / myos_tp as compiled from the header (gcc)
    against the ctypes mirrors: same size and field offsets."""
    import ctypes as C
    import shutil
    import subprocess
    if not shutil.which("gcc"):
        pytest.skip("gcc not available")
    structs = {"myos_shape": _lib.Shape, "myos_opts": _lib.Opts, "myos_tp": _lib.TP}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "myos_cuda.h"', "int main(void) {"]
    for cname, py in structs.items():
        lines.append('printf("%s %%zu\\n", sizeof(%s));' % (cname, cname))
        for field, _ in py._fields_:
            lines.append('printf("%s.%s %%zu\\n", offsetof(%s, %s));' % (cname, field, cname, field))
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run(["gcc", "-std=c11", "-I", os.path.join(REPO, "include"), str(src), "-o", str(exe)],
                   check=True)
    got = dict(l.split() for l in subprocess.run([str(exe)], capture_output=True, text=True,
                                                 check=True).stdout.splitlines())
    for cname, py in structs.items():
        assert int(got[cname]) == C.sizeof(py), cname
        for field, _ in py._fields_:
            assert int(got[f"{cname}.{field}"]) == getattr(py, field).offset, (cname, field)


def test_attention_argument_checks_need_no_gpu():
    """Both attention entry points refuse a mask kind other than Full (0) or
    Causal (1), and the no-allocation one refuses device pointers that are
    not 4-byte aligned, or K/V rows that are not 16-byte aligned when d % 4
    == 0, before any device work. The pointer values are never dereferenced:
    the checks return first, so no device is needed."""
    import ctypes as C
    L = _lib.load()
    hq, hkv, d, seq = 12, 2, 128, 16
    f = C.POINTER(C.c_float)
    y = np.zeros(hq * d, np.float32)
    q = np.zeros(hq * d, np.float32)
    k = np.zeros(hkv * seq * d, np.float32)
    for mask in (2, -1):
        st = L.myos_gqa_attn_f32(y.ctypes.data_as(f), y.size, q.ctypes.data_as(f), q.size,
                                 k.ctypes.data_as(f), k.size, k.ctypes.data_as(f), k.size,
                                 hq, hkv, d, seq, mask, 0)
        assert st == _lib.ERR_ARG, _lib.status_name(st)
    base = 1 << 40  # 256-byte aligned stand-in addresses
    ok = dict(d_y=base, d_q=base + 4096, d_k=base + 8192, d_v=base + (1 << 20))

    def noalloc(mask=0, dd=d, **over):
        p = dict(ok, **over)
        return L.myos_dev_gqa_attn_f32_noalloc(p["d_y"], p["d_q"], p["d_k"], p["d_v"], hq, hkv,
                                               dd, seq, mask, 0, None)

    assert noalloc(mask=2) == _lib.ERR_ARG
    assert noalloc(d_k=ok["d_k"] + 4) == _lib.ERR_ARG   # K rows not on 16 bytes
    assert noalloc(d_v=ok["d_v"] + 8) == _lib.ERR_ARG   # V rows not on 16 bytes
    assert noalloc(d_y=ok["d_y"] + 2) == _lib.ERR_ARG   # not even f32-aligned
    assert noalloc(d_q=ok["d_q"] + 1) == _lib.ERR_ARG
    # shape errors are reported before any device work as well
    assert noalloc(dd=0) == _lib.ERR_SHAPE
