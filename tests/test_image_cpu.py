"""Device images (foxcuda_model_save_image / foxcuda_model_open_image): the
checks that run before the device is touched, on image files written here
in the library's format.

A well-formed image passes every check and stops only at the device step
(no GPU in this container). Each damaged variant is refused with upstream's
status numbering: FOXCUDA_ERR_IO for a missing file, FOXCUDA_ERR_FORMAT for
a bad header, table or entry, FOXCUDA_ERR_UNSUPPORTED for another version.
"""
import ctypes
import struct

import pytest

import rustfox_b200 as rf
from rustfox_b200 import api

HEADER = struct.Struct("<8sIIQQIIII7I2f7I2f6I8IQ")
ENTRY = struct.Struct("<IIIIiiiiiiiiQQQQ")
EMBD, OUT_NORM, OUTPUT, ATTN_NORM, FFN_NORM, QKV, O, GATEUP, DOWN = range(9)
Q8_0, TQ2_0 = 8, 35


def fnv1a(b: bytes) -> int:
    h = 1469598103934665603
    for c in b:
        h = ((h ^ c) * 1099511628211) & (2**64 - 1)
    return h


def q8_bytes(rows, k):
    return rows * k // 32 * 34


def tq2_bytes(rows, k):
    return rows * k // 256 * 66


def image(n_layer=1, version=1, magic=b"FOXDIMG1", edit=None, truncate=0, table_hash=None):
    """A small model's image (hidden 256, 2/1 heads of 128, FFN 256, vocab
    64, TQ2_0 layers, Q8_0 embedding and head) with zero weights. `edit`
    may change the entry list before the table is hashed."""
    E, V, F_, nq, nkv = 256, 64, 256, 256, 128
    entries = []
    off = 0

    def add(kind, layer, index, nbytes, **kw):
        nonlocal off
        e = dict(kind=kind, layer=layer, index=index, flags=0, type=0, src_type=-1, n_rows=0, K=0, nb=0,
                 U=0, pro=1, qkv_base=0, ne0=0, ne1=0, offset=off, bytes=nbytes)
        e.update(kw)
        entries.append(e)
        off = (off + nbytes + 255) // 256 * 256

    add(EMBD, 0, 0, q8_bytes(V, E), type=Q8_0, ne0=E, ne1=V)
    add(OUT_NORM, 0, 0, E * 4)
    add(OUTPUT, 0, 0, q8_bytes(V, E), type=Q8_0, n_rows=V, K=E, nb=E // 32, U=32, flags=1)
    for l in range(n_layer):
        add(ATTN_NORM, l, 0, E * 4)
        add(FFN_NORM, l, 0, E * 4)
        add(QKV, l, 0, tq2_bytes(nq + 2 * nkv, E), type=TQ2_0, n_rows=nq + 2 * nkv, K=E, nb=1, U=64, pro=2)
        add(O, l, 0, tq2_bytes(E, nq), type=TQ2_0, n_rows=E, K=nq, nb=1, U=64)
        add(GATEUP, l, 0, tq2_bytes(2 * F_, E), type=TQ2_0, n_rows=2 * F_, K=E, nb=1, U=64, pro=2)
        add(DOWN, l, 0, tq2_bytes(E, F_), type=TQ2_0, n_rows=E, K=F_, nb=1, U=64)
    if edit:
        edit(entries)
    table = b"".join(ENTRY.pack(*(e[k] for k in ("kind", "layer", "index", "flags", "type", "src_type",
                                                  "n_rows", "K", "nb", "U", "pro", "qkv_base", "ne0",
                                                  "ne1", "offset", "bytes"))) for e in entries)
    data_off = (HEADER.size + len(table) + 4095) // 4096 * 4096
    info = (n_layer, E, 2, 1, F_, 128, V, 1e-5, 1e4)
    hdr = HEADER.pack(magic, version, len(entries), data_off, off, 148, 0, 1, 0, *info, *info,
                      0, 0, 0, nq // 256, 0, F_ // 256, F_ // 256, 0, 0, 0, 0, 0, 0, 0,
                      fnv1a(table) if table_hash is None else table_hash)
    blob = hdr + table + bytes(data_off - HEADER.size - len(table)) + bytes(off)
    return blob[:len(blob) - truncate] if truncate else blob


def open_status(path):
    h = ctypes.c_void_p()
    st = rf.lib().foxcuda_model_open_image(str(path).encode(), 0, ctypes.byref(h))
    assert not h.value
    return st, rf.last_error()


def test_record_sizes_match_the_library():
    assert HEADER.size == 184 and ENTRY.size == 80


def test_a_well_formed_image_passes_every_check_before_the_device(tmp_path):
    p = tmp_path / "ok.fdi"
    p.write_bytes(image(n_layer=2))
    st, msg = open_status(p)
    if st == api.OK:
        pytest.skip("a GPU is present: the GPU test opens real images")
    # refused only by the device step
    assert st not in (api.ERR_FORMAT, api.ERR_IO), msg
    assert "open_image" not in msg, msg


@pytest.mark.parametrize("case,want", [
    ("missing", api.ERR_IO),
    ("magic", api.ERR_FORMAT),
    ("version", api.ERR_UNSUPPORTED),
    ("truncated", api.ERR_FORMAT),
    ("hash", api.ERR_FORMAT),
    ("short_norm", api.ERR_FORMAT),
    ("wrong_shape", api.ERR_FORMAT),
    ("out_of_data", api.ERR_FORMAT),
    ("missing_down", api.ERR_FORMAT),
    ("repeated", api.ERR_FORMAT),
    ("qkv_rows", api.ERR_FORMAT),
    ("layer", api.ERR_FORMAT),
])
def test_damaged_images_are_refused_before_the_device(tmp_path, case, want):
    p = tmp_path / f"{case}.fdi"

    def edit_kind(kind, **kw):
        def f(entries):
            for e in entries:
                if e["kind"] == kind:
                    e.update(kw)
                    return
        return f

    blobs = {
        "magic": lambda: image(magic=b"GGUF\x03\x00\x00\x00"),
        "version": lambda: image(version=2),
        "truncated": lambda: image(truncate=100),
        "hash": lambda: image(table_hash=12345),
        "short_norm": lambda: image(edit=edit_kind(ATTN_NORM, bytes=1020)),
        "wrong_shape": lambda: image(edit=edit_kind(O, n_rows=128, bytes=tq2_bytes(128, 256))),
        "out_of_data": lambda: image(edit=edit_kind(DOWN, offset=1 << 30)),
        "missing_down": lambda: image(edit=lambda es: es.remove(next(e for e in es if e["kind"] == DOWN))),
        "repeated": lambda: image(edit=lambda es: es.append(dict(es[1]))),
        "qkv_rows": lambda: image(edit=edit_kind(QKV, n_rows=256, bytes=tq2_bytes(256, 256))),
        "layer": lambda: image(edit=edit_kind(FFN_NORM, layer=5)),
    }
    if case != "missing":
        p.write_bytes(blobs[case]())
    st, msg = open_status(p)
    assert st == want, msg
    assert "open_image" in msg


def test_save_checks_its_arguments():
    assert rf.lib().foxcuda_model_save_image(None, b"/nonexistent") == api.ERR_ARG
    assert rf.lib().foxcuda_model_get_info(None, None) == api.ERR_ARG
